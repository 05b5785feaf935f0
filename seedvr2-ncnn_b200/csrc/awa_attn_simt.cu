// awa_attn_simt.cu -- fp32 window attention on the CUDA cores, for the fp32
// DiT blocks (no TF32: every product and sum is an fp32 FFMA), and the general
// path for head_dim != 128.
//
// Math of SeedVR2WindowAttention::forward (awa_layers.cpp:1062-1120): for each
// window and head, softmax(Q K^T / sqrt(d)) V over the window's rows, no mask.
// Computed flash-style: one CTA per (window, 64-query tile, head), 64-key
// blocks, online softmax with exact running max, fp32 accumulation.
//
// Tiles: Q [128 d][64 rows] and K [128 d][64 keys] are stored d-major so both
// operands of the 4x4 register tile come as conflict-free float4 loads; V
// reuses the K buffer row-major once S is done; P is staged row-major.
// 81 KB of shared memory -> two CTAs per SM, which overlap one CTA's loads
// with the other's arithmetic.
#include "awa_rows.cuh"

#include <cuda_bf16.h>

namespace awa
{
namespace
{

using bf16 = __nv_bfloat16;

constexpr int BM = 64;
constexpr int BN = 64;
constexpr int D = 128;
constexpr int PS = BN + 4;  // P row stride (floats)
constexpr int kThreads = 256;

struct SimtShared
{
    float q[D * BM];
    float kv[D * BN];
    float p[BM * PS];
    int64_t q_dst[BM];       // output element offset of each query row (-1: invalid)
    int q_text[BM];          // query row is a text row (fused: goes to the text partials)
    const void* k_src[BN];   // q-segment pointer of each key row (nullptr: padding)
    int64_t k_step[BN];
    short4 k_coords[BN];
    const void* q_src[BM];
    int64_t q_step[BM];
    short4 q_coords[BM];
};

template <bool PACKED, typename TIn>
__device__ __forceinline__ void describe_rows(const AttnArgs& a, const WindowDesc& win, int first, int length,
                                              int count, int head, const void** src, int64_t* step, short4* coords)
{
    for (int r = threadIdx.x; r < count; r += kThreads)
    {
        const int row = first + r;
        if (row < length)
        {
            const RowRef ref = window_row<PACKED>(a, win, row, head);
            const TIn* base = PACKED ? static_cast<const TIn*>(a.qkv)
                                     : static_cast<const TIn*>(ref.is_text ? a.text_qkv : a.video_qkv);
            src[r] = base + ref.offset;
            step[r] = ref.qkv_step;
            coords[r] = ref.coords;
        }
        else
        {
            src[r] = nullptr;
            step[r] = 0;
            coords[r] = make_short4(0, 0, 0, 0);
        }
    }
}

// d-major tile [D][rows] of segment qkv (0 = Q, 1 = K), rotated when ROPE.
template <bool VEC, bool ROPE, typename TIn>
__device__ __forceinline__ void load_transposed(const AttnArgs& a, float* tile, const void* const* src,
                                                const int64_t* step, const short4* coords, int qkv)
{
    const int row = threadIdx.x & 63;
    const TIn* p = static_cast<const TIn*>(src[row]);
    const int hd = a.head_dim;
    if (VEC)
    {
        for (int c = threadIdx.x >> 6; c < D / 8; c += kThreads / 64)
        {
            float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            if (p && 8 * c < hd)
            {
                load8(p + qkv * step[row] + 8 * c, v);
                if (ROPE && a.rotate)
                    rope8(a.plan, coords[row], 8 * c, v);
            }
#pragma unroll
            for (int j = 0; j < 8; j++)
                tile[(8 * c + j) * 64 + row] = v[j];
        }
    }
    else
    {
        for (int f = threadIdx.x >> 6; f < D; f += kThreads / 64)
        {
            float v = 0.f;
            if (p && f < hd)
            {
                const TIn* seg = p + qkv * step[row];
                v = load1(seg + f);
                if (ROPE && a.rotate && f < a.plan.rope_dim)
                {
                    const float paired = load1(seg + (f ^ 1));
                    const float2 cs = rope_lookup(a.plan, coords[row], f >> 1);
                    float o0, o1;
                    if (f & 1)
                        rope_rotate(paired, v, cs.x, cs.y, o0, o1), v = o1;
                    else
                        rope_rotate(v, paired, cs.x, cs.y, o0, o1), v = o0;
                }
            }
            tile[f * 64 + row] = v;
        }
    }
}

// row-major V tile [BN][D]
template <bool VEC, typename TIn>
__device__ __forceinline__ void load_values(const AttnArgs& a, float* tile, const void* const* src, const int64_t* step)
{
    const int hd = a.head_dim;
    if (VEC)
    {
        for (int id = threadIdx.x; id < BN * D / 8; id += kThreads)
        {
            const int row = id >> 4;
            const int c = id & 15;
            const TIn* p = static_cast<const TIn*>(src[row]);
            float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            if (p && 8 * c < hd)
                load8(p + 2 * step[row] + 8 * c, v);
            float4* dst = reinterpret_cast<float4*>(tile + row * D + 8 * c);
            dst[0] = make_float4(v[0], v[1], v[2], v[3]);
            dst[1] = make_float4(v[4], v[5], v[6], v[7]);
        }
    }
    else
    {
        for (int id = threadIdx.x; id < BN * D; id += kThreads)
        {
            const int row = id / D;
            const int f = id - row * D;
            const TIn* p = static_cast<const TIn*>(src[row]);
            tile[id] = (p && f < hd) ? load1(p + 2 * step[row] + f) : 0.f;
        }
    }
}

template <typename T>
__device__ __forceinline__ void store4(T* dst, int col, int hd, float a0, float a1, float a2, float a3, bool vec)
{
    if (vec && col + 3 < hd)
    {
        if constexpr (sizeof(T) == 4)
            *reinterpret_cast<float4*>(dst + col) = make_float4(a0, a1, a2, a3);
        else
            *reinterpret_cast<uint2*>(dst + col) = make_uint2(pack_bf16x2(a0, a1), pack_bf16x2(a2, a3));
        return;
    }
    const float vals[4] = {a0, a1, a2, a3};
#pragma unroll
    for (int j = 0; j < 4; j++)
        if (col + j < hd)
            store1(dst + col + j, vals[j]);
}

// d += a * (b0, b1) on a register pair: sm_100 issues two fp32 FMAs per
// instruction (.f32x2); each lane rounds exactly as fmaf does, so the sums
// are the scalar loop's, bit for bit.
__device__ __forceinline__ void fma_bcast_x2(float& d0, float& d1, float a, float b0, float b1)
{
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %2};\n\t"
        "mov.b64 rb, {%3, %4};\n\t"
        "mov.b64 rd, {%0, %1};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rd;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "+f"(d0), "+f"(d1)
        : "f"(a), "f"(b0), "f"(b1));
}

template <bool PACKED, bool VEC, typename TIn, typename TOut>
__global__ void __launch_bounds__(kThreads, 2) attention_simt_kernel(const AttnArgs a)
{
    extern __shared__ float4 smem_raw[];
    SimtShared& sh = *reinterpret_cast<SimtShared*>(smem_raw);
    const int2 item = a.items[blockIdx.x];
    const int head = blockIdx.y;
    const WindowDesc win = a.plan.windows[item.x];
    const int text = a.plan.text_tokens;
    const int length = win.video + text;
    const int q0 = item.y * BM;
    const int tid = threadIdx.x;
    const int tr = tid >> 4;  // query rows 4tr .. 4tr+3
    const int tc = tid & 15;  // keys 4tc .. 4tc+3 ; output columns 4tc.., 64+4tc..
    const float scale_log2 = a.scale * 1.4426950408889634f;
    const int hd = a.head_dim;

    // Query rows: sources and output destinations.
    describe_rows<PACKED, TIn>(a, win, q0, length, BM, head, sh.q_src, sh.q_step, sh.q_coords);
    for (int r = tid; r < BM; r += kThreads)
    {
        const int row = q0 + r;
        int64_t dst = -1;
        int is_text = 0;
        if (row < length)
        {
            if (PACKED)
                dst = (int64_t)(win.offset + row) * a.out_token_stride + (int64_t)head * hd;
            else if (row < win.video)
                dst = window_row<false>(a, win, row, head).token * a.out_token_stride + (int64_t)head * hd;
            else
            {
                is_text = 1;
                const int slot = a.partial_slot ? a.partial_slot[item.x] : item.x - a.window_begin;
                dst = ((int64_t)slot * text + (row - win.video)) * a.heads * hd + (int64_t)head * hd;
            }
        }
        sh.q_dst[r] = dst;
        sh.q_text[r] = is_text;
    }
    __syncthreads();
    load_transposed<VEC, !PACKED, TIn>(a, sh.q, sh.q_src, sh.q_step, sh.q_coords, 0);

    float m[4], l[4], acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; i++)
    {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int j = 0; j < 8; j++)
            acc[i][j] = 0.f;
    }
    const int dmax = (hd + 3) & ~3;

    for (int k0 = 0; k0 < length; k0 += BN)
    {
        const int valid = min(BN, length - k0);
        __syncthreads();  // previous P / V reads are done
        describe_rows<PACKED, TIn>(a, win, k0, length, BN, head, sh.k_src, sh.k_step, sh.k_coords);
        __syncthreads();
        load_transposed<VEC, !PACKED, TIn>(a, sh.kv, sh.k_src, sh.k_step, sh.k_coords, 1);
        __syncthreads();

        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++)
                s[i][j] = 0.f;
#pragma unroll 4
        for (int f = 0; f < dmax; f++)
        {
            const float4 q = *reinterpret_cast<const float4*>(sh.q + f * BM + 4 * tr);
            const float4 k = *reinterpret_cast<const float4*>(sh.kv + f * BN + 4 * tc);
            const float qv[4] = {q.x, q.y, q.z, q.w};
            const float kv[4] = {k.x, k.y, k.z, k.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j += 2)
                    fma_bcast_x2(s[i][j], s[i][j + 1], qv[i], kv[j], kv[j + 1]);
        }

        // Online softmax over this key block (rows shared by the 16 lanes of a half-warp).
#pragma unroll
        for (int i = 0; i < 4; i++)
        {
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; j++)
            {
                s[i][j] = (4 * tc + j < valid) ? s[i][j] * scale_log2 : -INFINITY;
                mx = fmaxf(mx, s[i][j]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1)
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float m_new = fmaxf(m[i], mx);
            const float alpha = fast_exp2(m[i] - m_new);
            float sum = 0.f;
#pragma unroll
            for (int j = 0; j < 4; j++)
            {
                s[i][j] = (4 * tc + j < valid) ? fast_exp2(s[i][j] - m_new) : 0.f;
                sum += s[i][j];
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1)
                sum += __shfl_xor_sync(0xffffffffu, sum, off);
            l[i] = l[i] * alpha + sum;
            m[i] = m_new;
#pragma unroll
            for (int j = 0; j < 8; j++)
                acc[i][j] *= alpha;
            *reinterpret_cast<float4*>(sh.p + (4 * tr + i) * PS + 4 * tc) = make_float4(s[i][0], s[i][1], s[i][2], s[i][3]);
        }
        __syncthreads();  // K reads done, P visible
        load_values<VEC, TIn>(a, sh.kv, sh.k_src, sh.k_step);
        __syncthreads();

        const int kmax = (valid + 3) & ~3;
        for (int kk = 0; kk < kmax; kk += 4)
        {
            float4 p4[4];
#pragma unroll
            for (int i = 0; i < 4; i++)
                p4[i] = *reinterpret_cast<const float4*>(sh.p + (4 * tr + i) * PS + kk);
#pragma unroll
            for (int u = 0; u < 4; u++)
            {
                const float4 va = *reinterpret_cast<const float4*>(sh.kv + (kk + u) * D + 4 * tc);
                const float4 vb = *reinterpret_cast<const float4*>(sh.kv + (kk + u) * D + 64 + 4 * tc);
                const float vv[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};
#pragma unroll
                for (int i = 0; i < 4; i++)
                {
                    const float pv = u == 0 ? p4[i].x : u == 1 ? p4[i].y : u == 2 ? p4[i].z : p4[i].w;
#pragma unroll
                    for (int j = 0; j < 8; j += 2)
                        fma_bcast_x2(acc[i][j], acc[i][j + 1], pv, vv[j], vv[j + 1]);
                }
            }
        }
    }

    // Epilogue: normalise and write each valid query row.
#pragma unroll
    for (int i = 0; i < 4; i++)
    {
        const int r = 4 * tr + i;
        const int64_t dst = sh.q_dst[r];
        if (dst < 0)
            continue;
        const float inv = 1.f / l[i];
        if (!PACKED && sh.q_text[r])
        {
            float* out = a.text_partial + dst;
            store4(out, 4 * tc, hd, acc[i][0] * inv, acc[i][1] * inv, acc[i][2] * inv, acc[i][3] * inv, VEC);
            store4(out, 64 + 4 * tc, hd, acc[i][4] * inv, acc[i][5] * inv, acc[i][6] * inv, acc[i][7] * inv, VEC);
        }
        else
        {
            TOut* out = static_cast<TOut*>(a.out) + dst;
            store4(out, 4 * tc, hd, acc[i][0] * inv, acc[i][1] * inv, acc[i][2] * inv, acc[i][3] * inv, VEC);
            store4(out, 64 + 4 * tc, hd, acc[i][4] * inv, acc[i][5] * inv, acc[i][6] * inv, acc[i][7] * inv, VEC);
        }
    }
}

bool aligned16(const void* p)
{
    return (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

template <bool PACKED, bool VEC, typename TIn, typename TOut>
int launch_simt(const AttnArgs& a, cudaStream_t stream)
{
    const size_t smem = sizeof(SimtShared);
    auto kernel = attention_simt_kernel<PACKED, VEC, TIn, TOut>;
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
    // 8-element vector loads / 4-element vector stores need aligned rows.
    const size_t in = sizeof(TIn), out = sizeof(TOut);
    bool vec = a.head_dim % 8 == 0 && aligned16(a.out) && (a.out_token_stride * out) % 16 == 0;
    if (packed)
        vec = vec && aligned16(a.qkv) && (a.qkv_token_stride * in) % 16 == 0 && (a.heads * a.head_dim * in) % 16 == 0;
    else
        vec = vec && aligned16(a.video_qkv) && aligned16(a.text_qkv) && (a.video_token_stride * in) % 16 == 0 &&
              (a.video_qkv_stride * in) % 16 == 0 && (a.text_token_stride * in) % 16 == 0 &&
              (a.text_qkv_stride * in) % 16 == 0 && aligned16(a.text_partial);
    if (packed)
        return vec ? launch_simt<true, true, TIn, TOut>(a, stream) : launch_simt<true, false, TIn, TOut>(a, stream);
    return vec ? launch_simt<false, true, TIn, TOut>(a, stream) : launch_simt<false, false, TIn, TOut>(a, stream);
}

}  // namespace

int launch_attention_simt(const AttnArgs& args, int packed, int in_dtype, int out_dtype, cudaStream_t stream)
{
    ProfileScope prof(packed ? "awa_attention_simt_packed" : "awa_attention_simt_fused", stream);
    if (in_dtype == kF32 && out_dtype == kF32)
        return launch_typed<float, float>(args, packed, stream);
    if (in_dtype == kF32 && out_dtype == kBF16)
        return launch_typed<float, bf16>(args, packed, stream);
    if (in_dtype == kBF16 && out_dtype == kF32)
        return launch_typed<bf16, float>(args, packed, stream);
    return launch_typed<bf16, bf16>(args, packed, stream);
}

}  // namespace awa
