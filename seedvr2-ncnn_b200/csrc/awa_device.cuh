// awa_device.cuh -- small device helpers shared by the AWA kernels.
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

namespace awa
{

__device__ __forceinline__ float bf16_bits_to_float(uint32_t bits16)
{
    return __uint_as_float(bits16 << 16);
}

// Round-to-nearest-even fp32 -> bf16 pair packed low/high.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi)
{
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// 8 consecutive elements <-> 8 floats. Pointers must be 16-byte aligned.
__device__ __forceinline__ void load8(const float* p, float (&v)[8])
{
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8])
{
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; i++)
    {
        v[2 * i] = bf16_bits_to_float(w[i] & 0xffffu);
        v[2 * i + 1] = bf16_bits_to_float(w[i] >> 16);
    }
}

__device__ __forceinline__ void store8(float* p, const float (&v)[8])
{
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&v)[8])
{
    *reinterpret_cast<uint4*>(p) =
        make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
}

__device__ __forceinline__ float load1(const float* p)
{
    return __ldg(p);
}

__device__ __forceinline__ float load1(const __nv_bfloat16* p)
{
    return __bfloat162float(*p);
}

__device__ __forceinline__ void store1(float* p, float v)
{
    *p = v;
}

__device__ __forceinline__ void store1(__nv_bfloat16* p, float v)
{
    *p = __float2bfloat16_rn(v);
}

// Raw 16-byte copies when no conversion is needed.
template <typename T>
struct Elem8
{
    static constexpr int kBytes = 8 * sizeof(T);
};

}  // namespace awa
