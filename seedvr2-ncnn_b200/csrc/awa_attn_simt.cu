// awa_attn_simt.cu -- fp32 window attention on the CUDA cores, for the fp32
// DiT blocks (no TF32: every product and sum is an fp32 FFMA), and the general
// path for head_dim != 128.
//
// Math of SeedVR2WindowAttention::forward (awa_layers.cpp:1062-1120): for each
// window and head, softmax(Q K^T / sqrt(d)) V over the window's rows, no mask.
// Computed flash-style over 64-key blocks, online softmax with exact running
// max, fp32 accumulation. A work item is (window, 128-query tile); two
// kernels:
//
// * attention_simt_async_kernel (fp32 rows, head_dim 128, 16-byte aligned):
//   one CTA of 512 threads per (item, head). Q, K and V rows are copied as
//   they lie (row-major, 132-float stride) by cp.async, two K/V stages, so
//   block j + 1 streams in while block j is computed; Q and K are rotated in
//   place in shared memory. Each thread holds a 4 (rows) x 4 (keys) score tile
//   and a 4 x 8 output tile; S runs as two partial sums (even and odd
//   features) on packed pairs, P overlays the finished K stage. 201 KB of
//   shared memory, one CTA per SM.
// * attention_simt_kernel (the general path: bf16 rows, other head sizes,
//   unaligned rows): one CTA of 256 threads per (item half of 64 rows, head).
//   Q [128 d][64 rows] and K [128 d][64 keys] are stored d-major so both
//   operands of the 4x4 register tile come as conflict-free float4 loads; V
//   reuses the K buffer row-major once S is done; P is staged row-major. 81 KB
//   of shared memory -> two CTAs per SM, which overlap one CTA's loads with the
//   other's arithmetic.
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
    const int2 item = a.items[blockIdx.x >> 1];
    const int head = blockIdx.y;
    const WindowDesc win = a.plan.windows[item.x];
    const int text = a.plan.text_tokens;
    const int length = win.video + text;
    const int q0 = item.y * kSimtRowsPerTile + (blockIdx.x & 1) * BM;  // this CTA's half of the item
    if (q0 >= length)
        return;
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

// ---- fp32 rows, head_dim 128: cp.async staging, 128-row tiles ----

constexpr int kAsyncRows = 128;    // query rows of a CTA (= kSimtRowsPerTile)
constexpr int kAsyncKeys = 64;     // keys of a block
constexpr int kAsyncLd = 132;      // row stride of the Q/K/V tiles (floats): 16-byte rows, conflict-free key columns
constexpr int kAsyncPs = 64;       // P row stride (floats)
constexpr int kAsyncThreads = 512;

struct AsyncShared
{
    float q[kAsyncRows * kAsyncLd];
    float k[2][kAsyncKeys * kAsyncLd];  // P [BM][PS] overlays the stage of the block being finished
    float v[2][kAsyncKeys * kAsyncLd];
    int64_t q_dst[kAsyncRows];  // output element offset of each query row (-1: invalid)
    int q_text[kAsyncRows];     // query row is a text row (fused: goes to the text partials)
    short4 k_coords[2][kAsyncKeys];
};
static_assert(kAsyncRows * kAsyncPs <= kAsyncKeys * kAsyncLd, "P must fit in a K stage");
static_assert(kAsyncRows == kSimtRowsPerTile, "a CTA takes one work item");

// 16 bytes global -> shared without registers; valid == false fills zeros
// (src-size 0: nothing is read).
__device__ __forceinline__ void cp_async16(float* smem, const float* gmem, bool valid)
{
    const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(gmem), "r"(valid ? 16 : 0)
                 : "memory");
}

__device__ __forceinline__ void cp_async_commit()
{
    asm volatile("cp.async.commit_group;\n" ::: "memory");
}

// Waits until at most one committed group of this thread is still in flight.
__device__ __forceinline__ void cp_async_wait_all_but_one()
{
    asm volatile("cp.async.wait_group 1;\n" ::: "memory");
}

// (d0, d1) += (a0, a1) * (b0, b1) in one packed instruction, each lane rounded
// as fmaf.
__device__ __forceinline__ void fma_x2(float& d0, float& d1, float a0, float a1, float b0, float b1)
{
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %5};\n\t"
        "mov.b64 rd, {%0, %1};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rd;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "+f"(d0), "+f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// Rotates the pairs first, first + stride, ... (< rope_dim / 2) of one row in
// shared memory with the reference's rotation (rope_rotate).
__device__ __forceinline__ void rotate_row(const PlanDevice& plan, float* row, short4 coords, int first, int stride)
{
    const int pairs = plan.rope_dim >> 1;
    for (int p = first; p < pairs; p += stride)
    {
        float2* x = reinterpret_cast<float2*>(row + 2 * p);
        const float2 v = *x;
        const float2 cs = rope_lookup(plan, coords, p);
        float o0, o1;
        rope_rotate(v.x, v.y, cs.x, cs.y, o0, o1);
        *x = make_float2(o0, o1);
    }
}

// Issues the copies of K/V block rows [k0, k0 + 64) into one stage: thread t
// takes row t / 8 and its 16-byte chunks t % 8 + 8m. Rows past the window are
// zero-filled.
template <bool PACKED>
__device__ __forceinline__ void issue_kv(const AttnArgs& a, const WindowDesc& win, int length, int head, int k0,
                                         float* kdst, float* vdst, short4* coords)
{
    const int r = threadIdx.x >> 3;
    const int part = threadIdx.x & 7;
    const int row = k0 + r;
    const bool ok = row < length;
    const float* src = static_cast<const float*>(PACKED ? a.qkv : a.video_qkv);
    int64_t step = 0;
    short4 c = make_short4(0, 0, 0, 0);
    if (ok)
    {
        const RowRef ref = window_row<PACKED>(a, win, row, head);
        if (!PACKED && ref.is_text)
            src = static_cast<const float*>(a.text_qkv);
        src += ref.offset;
        step = ref.qkv_step;
        c = ref.coords;
    }
    if (part == 0)
        coords[r] = c;
#pragma unroll
    for (int m = 0; m < 4; m++)
    {
        const int f = 4 * (part + 8 * m);
        cp_async16(kdst + r * kAsyncLd + f, src + step + f, ok);
        cp_async16(vdst + r * kAsyncLd + f, src + 2 * step + f, ok);
    }
}

template <bool PACKED, typename TOut>
__global__ void __launch_bounds__(kAsyncThreads, 1) attention_simt_async_kernel(const AttnArgs a)
{
    extern __shared__ float4 smem_raw[];
    AsyncShared& sh = *reinterpret_cast<AsyncShared*>(smem_raw);
    const int2 item = a.items[blockIdx.x];
    const int head = blockIdx.y;
    const WindowDesc win = a.plan.windows[item.x];
    const int text = a.plan.text_tokens;
    const int length = win.video + text;
    const int q0 = item.y * kAsyncRows;
    const int tid = threadIdx.x;
    const int tr = tid >> 4;  // query rows 4tr .. 4tr+3
    const int tc = tid & 15;  // keys tc + 16j ; output columns 4tc.., 64+4tc..
    const float scale_log2 = a.scale * 1.4426950408889634f;
    constexpr int D = 128;
    const bool rotate = !PACKED && a.rotate;
    // warps whose eight query rows all lie past the window skip the arithmetic
    const bool active = 8 * (tid >> 5) < length - q0;

    // Q rows (thread t: row t / 4, chunks t % 4 + 4m) and their destinations.
    const int qr = tid >> 2;
    short4 q_coords = make_short4(0, 0, 0, 0);
    {
        const int row = q0 + qr;
        const bool ok = row < length;
        const float* src = static_cast<const float*>(PACKED ? a.qkv : a.video_qkv);
        int64_t dst = -1;
        int is_text = 0;
        if (ok)
        {
            const RowRef ref = window_row<PACKED>(a, win, row, head);
            if (!PACKED && ref.is_text)
                src = static_cast<const float*>(a.text_qkv);
            src += ref.offset;
            q_coords = ref.coords;
            if (PACKED)
                dst = (int64_t)(win.offset + row) * a.out_token_stride + (int64_t)head * D;
            else if (!ref.is_text)
                dst = ref.token * a.out_token_stride + (int64_t)head * D;
            else
            {
                is_text = 1;
                const int slot = a.partial_slot ? a.partial_slot[item.x] : item.x - a.window_begin;
                dst = ((int64_t)slot * text + ref.text_index) * a.heads * D + (int64_t)head * D;
            }
        }
        if ((tid & 3) == 0)
        {
            sh.q_dst[qr] = dst;
            sh.q_text[qr] = is_text;
        }
#pragma unroll
        for (int m = 0; m < 8; m++)
        {
            const int f = 4 * ((tid & 3) + 4 * m);
            cp_async16(sh.q + qr * kAsyncLd + f, src + f, ok);
        }
    }
    issue_kv<PACKED>(a, win, length, head, 0, sh.k[0], sh.v[0], sh.k_coords[0]);
    cp_async_commit();
    issue_kv<PACKED>(a, win, length, head, kAsyncKeys, sh.k[1], sh.v[1], sh.k_coords[1]);  // zero rows if past the window
    cp_async_commit();

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

    for (int k0 = 0, st = 0; k0 < length; k0 += kAsyncKeys, st ^= 1)
    {
        const int valid = min(kAsyncKeys, length - k0);
        float* kst = sh.k[st];
        const float* vst = sh.v[st];
        cp_async_wait_all_but_one();  // this block's rows (and Q) have landed
        __syncthreads();
        if (rotate)
        {
            if (k0 == 0 && q0 + qr < length)
                rotate_row(a.plan, sh.q + qr * kAsyncLd, q_coords, tid & 3, 4);
            if (k0 + (tid >> 3) < length)
                rotate_row(a.plan, kst + (tid >> 3) * kAsyncLd, sh.k_coords[st][tid >> 3], tid & 7, 8);
            __syncthreads();
        }

        float s[4][4];
        if (active)
        {
            float se[4][4], so[4][4];  // partial sums over even / odd features
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++)
                    se[i][j] = so[i][j] = 0.f;
            const float* qrow = sh.q + 4 * tr * kAsyncLd;
            const float* krow = kst + tc * kAsyncLd;
#pragma unroll 2
            for (int f = 0; f < D; f += 4)
            {
                float4 kv[4];
#pragma unroll
                for (int j = 0; j < 4; j++)
                    kv[j] = *reinterpret_cast<const float4*>(krow + 16 * j * kAsyncLd + f);
#pragma unroll
                for (int i = 0; i < 4; i++)
                {
                    const float4 q = *reinterpret_cast<const float4*>(qrow + i * kAsyncLd + f);
#pragma unroll
                    for (int j = 0; j < 4; j++)
                    {
                        fma_x2(se[i][j], so[i][j], q.x, q.y, kv[j].x, kv[j].y);
                        fma_x2(se[i][j], so[i][j], q.z, q.w, kv[j].z, kv[j].w);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++)
                    s[i][j] = se[i][j] + so[i][j];
        }
        __syncthreads();  // every read of this K stage is done: P overlays it

        float* P = kst;
        if (active)
        {
#pragma unroll
            for (int i = 0; i < 4; i++)
            {
                float mx = -INFINITY;
#pragma unroll
                for (int j = 0; j < 4; j++)
                {
                    s[i][j] = (tc + 16 * j < valid) ? s[i][j] * scale_log2 : -INFINITY;
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
                    s[i][j] = (tc + 16 * j < valid) ? fast_exp2(s[i][j] - m_new) : 0.f;
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
#pragma unroll
                for (int j = 0; j < 4; j++)
                    P[(4 * tr + i) * kAsyncPs + tc + 16 * j] = s[i][j];
            }
        }
        __syncthreads();  // P visible

        if (active)
        {
            const int kmax = (valid + 3) & ~3;
            const float* prow = P + 4 * tr * kAsyncPs;
            for (int kk = 0; kk < kmax; kk += 4)
            {
                float4 p4[4];
#pragma unroll
                for (int i = 0; i < 4; i++)
                    p4[i] = *reinterpret_cast<const float4*>(prow + i * kAsyncPs + kk);
#pragma unroll
                for (int u = 0; u < 4; u++)
                {
                    const float4 va = *reinterpret_cast<const float4*>(vst + (kk + u) * kAsyncLd + 4 * tc);
                    const float4 vb = *reinterpret_cast<const float4*>(vst + (kk + u) * kAsyncLd + 64 + 4 * tc);
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
        __syncthreads();  // P and V reads are done: the stage takes block + 2
        if (k0 + 2 * kAsyncKeys < length)
            issue_kv<PACKED>(a, win, length, head, k0 + 2 * kAsyncKeys, sh.k[st], sh.v[st], sh.k_coords[st]);
        cp_async_commit();  // (an empty group past the last block keeps the count uniform)
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
            store4(out, 4 * tc, D, acc[i][0] * inv, acc[i][1] * inv, acc[i][2] * inv, acc[i][3] * inv, true);
            store4(out, 64 + 4 * tc, D, acc[i][4] * inv, acc[i][5] * inv, acc[i][6] * inv, acc[i][7] * inv, true);
        }
        else
        {
            TOut* out = static_cast<TOut*>(a.out) + dst;
            store4(out, 4 * tc, D, acc[i][0] * inv, acc[i][1] * inv, acc[i][2] * inv, acc[i][3] * inv, true);
            store4(out, 64 + 4 * tc, D, acc[i][4] * inv, acc[i][5] * inv, acc[i][6] * inv, acc[i][7] * inv, true);
        }
    }
}

template <bool PACKED, typename TOut>
int launch_async(const AttnArgs& a, cudaStream_t stream)
{
    const size_t smem = sizeof(AsyncShared);
    auto kernel = attention_simt_async_kernel<PACKED, TOut>;
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess)
        return (int)err;
    dim3 grid(a.item_count, a.heads);
    kernel<<<grid, kAsyncThreads, smem, stream>>>(a);
    return (int)cudaGetLastError();
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
    dim3 grid(2 * a.item_count, a.heads);
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
    if constexpr (sizeof(TIn) == 4)
        if (vec && a.head_dim == D)
            return packed ? launch_async<true, TOut>(a, stream) : launch_async<false, TOut>(a, stream);
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
