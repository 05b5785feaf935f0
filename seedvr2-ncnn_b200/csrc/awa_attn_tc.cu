// awa_attn_tc.cu -- bf16 window attention on the sm_100a tensor cores
// (tcgen05.mma, fp32 accumulators in TMEM), for the bf16 DiT blocks.
//
// Math of SeedVR2WindowAttention::forward (awa_layers.cpp:1062-1120): per
// window and head, softmax(Q K^T / sqrt(d)) V over the window rows. One CTA of
// 4 warps takes one (window, 128-query tile, head) work item:
//
//   Q tile (128 x 128 bf16) and each 128-key block of K and V are staged in
//   shared memory in the 128-byte-swizzled K-major layout the tensor core
//   reads (rows of 128 B, 16-byte chunks XOR-permuted by row % 8). In fused
//   mode the rows are gathered straight from the source QKV by window
//   geometry and Q/K are rotated (3D RoPE) between the global load and the
//   shared store, so the packed layout is never written to HBM.
//
//   S = Q K^T       tcgen05.mma, A and B from shared memory, D in TMEM
//                   columns 0..127 (one lane per query row).
//   softmax         each thread owns one row: tcgen05.ld of its S row, online
//                   max (rescaling O only when the max grows by more than
//                   2^8), exp2, P rounded to bf16 and written back over S in
//                   TMEM (tcgen05.st, two P values per 32-bit column).
//   O += P V        tcgen05.mma with A = P from TMEM, B = V (MN-major view of
//                   the same swizzled tile), D = O in TMEM columns 128..255.
//   epilogue        O / l, converted, each thread stores its row.
//
// 256 TMEM columns and ~100 KB of shared memory per CTA: two CTAs per SM, so
// one CTA's loads and softmax overlap the other's MMAs.
#include "awa_rows.cuh"
#include "tcgen05.cuh"

#include <cuda_bf16.h>

namespace awa
{
namespace
{

using bf16 = __nv_bfloat16;

constexpr int kRows = 128;                    // query rows per tile = keys per block
constexpr int kHeadDim = 128;
constexpr int kPanelBytes = kRows * 128;      // 64 bf16 features x 128 rows
constexpr int kTileBytes = 2 * kPanelBytes;   // 128 x 128 bf16
constexpr int kThreads = 128;
constexpr uint32_t kTmemColumns = 256;
constexpr uint32_t kColS = 0;    // S (fp32) / P (bf16 pairs) columns
constexpr uint32_t kColO = 128;  // O accumulator columns

struct TcRows
{
    const void* src[kRows];
    int64_t step[kRows];
    short4 coords[kRows];
};

struct TcShared
{
    uint8_t q[kTileBytes];
    uint8_t k[kTileBytes];
    uint8_t v[kTileBytes];
    TcRows q_rows;
    TcRows k_rows;
    int64_t q_dst[kRows];
    int q_text[kRows];
    uint64_t bar;
    uint32_t tmem_base;
    int abort;
};

template <typename T>
struct Raw8;
template <>
struct Raw8<bf16>
{
    uint4 u;
};
template <>
struct Raw8<float>
{
    float4 a, b;
};

__device__ __forceinline__ Raw8<bf16> load_raw(const bf16* p)
{
    return {__ldg(reinterpret_cast<const uint4*>(p))};
}
__device__ __forceinline__ Raw8<float> load_raw(const float* p)
{
    return {__ldg(reinterpret_cast<const float4*>(p)), __ldg(reinterpret_cast<const float4*>(p) + 1)};
}
__device__ __forceinline__ void zero_raw(Raw8<bf16>& r)
{
    r.u = make_uint4(0, 0, 0, 0);
}
__device__ __forceinline__ void zero_raw(Raw8<float>& r)
{
    r.a = r.b = make_float4(0.f, 0.f, 0.f, 0.f);
}
__device__ __forceinline__ void unpack_raw(const Raw8<bf16>& r, float (&v)[8])
{
    const uint32_t w[4] = {r.u.x, r.u.y, r.u.z, r.u.w};
#pragma unroll
    for (int i = 0; i < 4; i++)
    {
        v[2 * i] = bf16_bits_to_float(w[i] & 0xffffu);
        v[2 * i + 1] = bf16_bits_to_float(w[i] >> 16);
    }
}
__device__ __forceinline__ void unpack_raw(const Raw8<float>& r, float (&v)[8])
{
    v[0] = r.a.x; v[1] = r.a.y; v[2] = r.a.z; v[3] = r.a.w;
    v[4] = r.b.x; v[5] = r.b.y; v[6] = r.b.z; v[7] = r.b.w;
}

// Byte offset of 16-byte chunk c (0..15 along the 128 features) of row r in
// a swizzled tile: two 64-feature panels, 128-byte rows, chunk index XOR row%8.
__device__ __forceinline__ uint32_t swizzled_offset(int r, int c)
{
    return (uint32_t)((c >> 3) * kPanelBytes + r * 128 + ((((c & 7) ^ (r & 7))) << 4));
}

template <bool PACKED, typename TIn>
__device__ __forceinline__ void describe_rows(const AttnArgs& a, const WindowDesc& win, int first, int length,
                                              int head, TcRows& rows)
{
    const int r = threadIdx.x;  // one row per thread
    const int row = first + r;
    if (row < length)
    {
        const RowRef ref = window_row<PACKED>(a, win, row, head);
        const TIn* base =
            PACKED ? static_cast<const TIn*>(a.qkv) : static_cast<const TIn*>(ref.is_text ? a.text_qkv : a.video_qkv);
        rows.src[r] = base + ref.offset;
        rows.step[r] = ref.qkv_step;
        rows.coords[r] = ref.coords;
    }
    else
    {
        rows.src[r] = nullptr;
        rows.step[r] = 0;
        rows.coords[r] = make_short4(0, 0, 0, 0);
    }
}

// Load segment `qkv` of 128 rows into a swizzled bf16 tile; rows without a
// source are zero. 16 threads cover one 256-byte row (coalesced); the loads of
// a batch are all issued before any is consumed.
template <bool ROPE, typename TIn>
__device__ __forceinline__ void load_tile(const AttnArgs& a, uint8_t* tile, const TcRows& rows, int qkv)
{
    constexpr int kBatch = sizeof(TIn) == 2 ? 16 : 8;
    const int c = threadIdx.x & 15;
    const int r0 = threadIdx.x >> 4;
#pragma unroll
    for (int j0 = 0; j0 < 16; j0 += kBatch)
    {
        Raw8<TIn> raw[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; j++)
        {
            const int r = r0 + 8 * (j0 + j);
            const TIn* p = static_cast<const TIn*>(rows.src[r]);
            if (p)
                raw[j] = load_raw(p + qkv * rows.step[r] + 8 * c);
            else
                zero_raw(raw[j]);
        }
#pragma unroll
        for (int j = 0; j < kBatch; j++)
        {
            const int r = r0 + 8 * (j0 + j);
            float v[8];
            unpack_raw(raw[j], v);
            if (ROPE)
                rope8(a.plan, rows.coords[r], 8 * c, v);
            *reinterpret_cast<uint4*>(tile + swizzled_offset(r, c)) =
                make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                           pack_bf16x2(v[6], v[7]));
        }
    }
}

// S[128 x n] = Q K^T over the 128 features (8 MMAs of K = 16).
__device__ __forceinline__ void issue_qk(uint32_t tmem_s, uint32_t q_addr, uint32_t k_addr, int n)
{
    const uint32_t idesc = tc::idesc_bf16_f32(128, n, false);
#pragma unroll
    for (int ks = 0; ks < 8; ks++)
    {
        const uint32_t off = (uint32_t)((ks >> 2) * kPanelBytes + (ks & 3) * 32);
        tc::mma_ss(tmem_s, tc::smem_desc_sw128(q_addr + off, 16, 1024), tc::smem_desc_sw128(k_addr + off, 16, 1024),
                   idesc, ks > 0 ? 1u : 0u);
    }
}

// O[128 x 128] (+)= P[128 x n] V[n x 128]; P in TMEM (bf16 pairs), V MN-major:
// 8-key groups 1024 B apart (SBO), 64-feature panels kPanelBytes apart (LBO).
__device__ __forceinline__ void issue_pv(uint32_t tmem_o, uint32_t tmem_p, uint32_t v_addr, int n, bool accumulate)
{
    const uint32_t idesc = tc::idesc_bf16_f32(128, 128, true);
    for (int ks = 0; ks < n / 16; ks++)
        tc::mma_ts(tmem_o, tmem_p + (uint32_t)(ks * 8), tc::smem_desc_sw128(v_addr + (uint32_t)(ks * 2048), kPanelBytes, 1024),
                   idesc, (accumulate || ks > 0) ? 1u : 0u);
}

template <typename T>
__device__ __forceinline__ void store_row32(T* dst, const float (&v)[32]);

template <>
__device__ __forceinline__ void store_row32<float>(float* dst, const float (&v)[32])
{
#pragma unroll
    for (int i = 0; i < 8; i++)
        reinterpret_cast<float4*>(dst)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

template <>
__device__ __forceinline__ void store_row32<bf16>(bf16* dst, const float (&v)[32])
{
#pragma unroll
    for (int i = 0; i < 4; i++)
        reinterpret_cast<uint4*>(dst)[i] =
            make_uint4(pack_bf16x2(v[8 * i], v[8 * i + 1]), pack_bf16x2(v[8 * i + 2], v[8 * i + 3]),
                       pack_bf16x2(v[8 * i + 4], v[8 * i + 5]), pack_bf16x2(v[8 * i + 6], v[8 * i + 7]));
}

template <bool PACKED, typename TIn, typename TOut>
__global__ void __launch_bounds__(kThreads, 2) attention_tc_kernel(const AttnArgs a)
{
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the 128-byte swizzle atoms.
    const uint32_t raw_addr = tc::smem_addr(smem_raw);
    TcShared& sh = *reinterpret_cast<TcShared*>(smem_raw + ((1024 - (raw_addr & 1023)) & 1023));

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int2 item = a.items[blockIdx.x];
    const int head = blockIdx.y;
    const WindowDesc win = a.plan.windows[item.x];
    const int text = a.plan.text_tokens;
    const int length = win.video + text;
    const int q0 = item.y * kRows;
    const float scale_log2 = a.scale * 1.4426950408889634f;

    if (warp == 0)
    {
        tc::tmem_alloc(&sh.tmem_base, kTmemColumns);
        tc::tmem_relinquish();
    }
    if (tid == 0)
    {
        tc::mbar_init(&sh.bar, 1);
        tc::mbar_fence_init();
        sh.abort = 0;
    }
    // Query rows: sources and destinations.
    describe_rows<PACKED, TIn>(a, win, q0, length, head, sh.q_rows);
    {
        const int row = q0 + tid;
        int64_t dst = -1;
        int is_text = 0;
        if (row < length)
        {
            if (PACKED)
                dst = (int64_t)(win.offset + row) * a.out_token_stride + (int64_t)head * kHeadDim;
            else if (row < win.video)
                dst = window_row<false>(a, win, row, head).token * a.out_token_stride + (int64_t)head * kHeadDim;
            else
            {
                is_text = 1;
                dst = ((int64_t)(item.x - a.window_begin) * text + (row - win.video)) * a.heads * kHeadDim +
                      (int64_t)head * kHeadDim;
            }
        }
        sh.q_dst[tid] = dst;
        sh.q_text[tid] = is_text;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = sh.tmem_base;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const uint32_t q_addr = tc::smem_addr(sh.q);
    const uint32_t k_addr = tc::smem_addr(sh.k);
    const uint32_t v_addr = tc::smem_addr(sh.v);

    load_tile<!PACKED, TIn>(a, sh.q, sh.q_rows, 0);

    float m_run = -INFINITY;
    float l_run = 0.f;
    uint32_t phase = 0;
    bool ok = true;
    const int blocks = (length + kRows - 1) / kRows;
    for (int kb = 0; kb < blocks && ok; kb++)
    {
        const int k0 = kb * kRows;
        const int valid = min(kRows, length - k0);
        const int n = max(16, (valid + 15) & ~15);
        describe_rows<PACKED, TIn>(a, win, k0, length, head, sh.k_rows);
        __syncthreads();
        load_tile<!PACKED, TIn>(a, sh.k, sh.k_rows, 1);
        load_tile<false, TIn>(a, sh.v, sh.k_rows, 2);
        tc::fence_async_smem();  // generic-proxy stores -> tensor-core reads
        __syncthreads();
        if (tid == 0)
        {
            tc::fence_after_sync();
            issue_qk(tmem + kColS, q_addr, k_addr, n);
            tc::mma_commit(&sh.bar);
        }
        if (__syncthreads_or(!tc::mbar_wait(&sh.bar, phase, a.error_flag, 1)))
        {
            ok = false;
            break;
        }
        phase ^= 1;
        tc::fence_after_sync();

        // ---- softmax of this row over the block
        float s[kRows];
#pragma unroll
        for (int c = 0; c < kRows / 16; c++)
        {
            if (c * 16 < n)
            {
                uint32_t r[16];
                tc::tmem_ld16(tmem + lane_base + kColS + c * 16, r);
                tc::tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; j++)
                    s[c * 16 + j] = __uint_as_float(r[j]);
            }
        }
        float mb = -INFINITY;
#pragma unroll
        for (int j = 0; j < kRows; j++)
        {
            if (j < n)
            {
                s[j] = j < valid ? s[j] * scale_log2 : -INFINITY;
                mb = fmaxf(mb, s[j]);
            }
        }
        float alpha = 1.f;
        bool rescale = false;
        if (kb == 0)
            m_run = mb;
        else if (mb > m_run + 8.f)
        {
            alpha = fast_exp2(m_run - mb);
            m_run = mb;
            rescale = true;
        }
        float row_sum = 0.f;
#pragma unroll
        for (int c = 0; c < kRows / 16; c++)
        {
            if (c * 16 < n)
            {
                uint32_t pk[8];
#pragma unroll
                for (int i = 0; i < 8; i++)
                {
                    const float p0 = fast_exp2(s[c * 16 + 2 * i] - m_run);
                    const float p1 = fast_exp2(s[c * 16 + 2 * i + 1] - m_run);
                    pk[i] = pack_bf16x2(p0, p1);
                    row_sum += bf16_bits_to_float(pk[i] & 0xffffu) + bf16_bits_to_float(pk[i] >> 16);
                }
                tc::tmem_st8(tmem + lane_base + kColS + c * 8, pk);
            }
        }
        l_run = l_run * alpha + row_sum;
        if (__any_sync(0xffffffffu, rescale))
        {
#pragma unroll
            for (int c = 0; c < 4; c++)
            {
                uint32_t o[32];
                tc::tmem_ld32(tmem + lane_base + kColO + c * 32, o);
                tc::tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; j++)
                    o[j] = __float_as_uint(__uint_as_float(o[j]) * alpha);
                tc::tmem_st32(tmem + lane_base + kColO + c * 32, o);
            }
        }
        tc::tmem_wait_st();
        tc::fence_before_sync();
        __syncthreads();
        if (tid == 0)
        {
            tc::fence_after_sync();
            issue_pv(tmem + kColO, tmem + kColS, v_addr, n, kb > 0);
            tc::mma_commit(&sh.bar);
        }
        if (__syncthreads_or(!tc::mbar_wait(&sh.bar, phase, a.error_flag, 2)))
        {
            ok = false;
            break;
        }
        phase ^= 1;
        tc::fence_after_sync();
    }

    if (ok)
    {
        const int64_t dst = sh.q_dst[tid];
        const float inv = 1.f / l_run;
#pragma unroll
        for (int c = 0; c < 4; c++)
        {
            uint32_t o[32];
            tc::tmem_ld32(tmem + lane_base + kColO + c * 32, o);
            tc::tmem_wait_ld();
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; j++)
                v[j] = __uint_as_float(o[j]) * inv;
            if (dst >= 0)
            {
                if (!PACKED && sh.q_text[tid])
                    store_row32<float>(a.text_partial + dst + c * 32, v);
                else
                    store_row32<TOut>(static_cast<TOut*>(a.out) + dst + c * 32, v);
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0)
    {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemColumns);
    }
}

template <bool PACKED, typename TIn, typename TOut>
int launch_tc(const AttnArgs& a, cudaStream_t stream)
{
    const size_t smem = sizeof(TcShared) + 1024;
    auto kernel = attention_tc_kernel<PACKED, TIn, TOut>;
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess)
        return (int)err;
    dim3 grid(a.item_count, a.heads);
    kernel<<<grid, kThreads, smem, stream>>>(a);
    return (int)cudaGetLastError();
}

template <typename TIn, typename TOut>
int launch_typed(const AttnArgs& a, int packed, cudaStream_t stream)
{
    return packed ? launch_tc<true, TIn, TOut>(a, stream) : launch_tc<false, TIn, TOut>(a, stream);
}

}  // namespace

int launch_attention_tc(const AttnArgs& args, int packed, int in_dtype, int out_dtype, cudaStream_t stream)
{
    if (args.head_dim != kHeadDim)
        return (int)cudaErrorInvalidValue;
    ProfileScope prof(packed ? "awa_attention_tc_packed" : "awa_attention_tc_fused", stream);
    if (in_dtype == kF32 && out_dtype == kF32)
        return launch_typed<float, float>(args, packed, stream);
    if (in_dtype == kF32 && out_dtype == kBF16)
        return launch_typed<float, bf16>(args, packed, stream);
    if (in_dtype == kBF16 && out_dtype == kF32)
        return launch_typed<bf16, float>(args, packed, stream);
    return launch_typed<bf16, bf16>(args, packed, stream);
}

}  // namespace awa
