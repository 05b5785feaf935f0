// awa_copy_kernels.cu -- the HBM-bound layers of the AWA chain:
//   Pack      (awa_layers.cpp:419-458): gather source QKV rows into window order
//   MMRoPE    (awa_layers.cpp:913-953): rotate Q/K features in interleaved pairs
//   Unpack    (awa_layers.cpp:638-689): video rows back to source order, text mean
// plus the text reduction of the fused path and the shard copies of the
// multi-GPU path. Each thread moves 8 consecutive elements (16 or 32 bytes)
// when rows allow it, so warps issue full-sector, coalesced accesses; grids
// are sized in multiples of the SM count and stride over the work.
#include "awa_device.cuh"
#include "awa_internal.h"

#include <algorithm>

#include <cuda_bf16.h>

namespace awa
{
namespace
{

using bf16 = __nv_bfloat16;

int grid_for(int64_t work, int threads)
{
    static int sms = 0;
    if (sms == 0)
    {
        int device = 0;
        cudaGetDevice(&device);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        if (sms <= 0)
            sms = 148;
    }
    const int64_t blocks = (work + threads - 1) / threads;
    const int64_t cap = (int64_t)sms * 16;
    return (int)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

bool aligned16(const void* p)
{
    return (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

// 8-element chunks are usable when every chunk start is 16-byte aligned.
bool chunkable(int64_t row_elems, size_t elem, const void* const* ptrs, int nptr, const int64_t* strides, int nstride)
{
    if (row_elems % 8)
        return false;
    for (int i = 0; i < nptr; i++)
        if (!aligned16(ptrs[i]))
            return false;
    for (int i = 0; i < nstride; i++)
        if ((strides[i] * (int64_t)elem) % 16)
            return false;
    return true;
}

// ---------------------------------------------------------------- Pack
template <typename TIn, typename TOut>
__global__ void pack_chunks(PlanDevice plan, int head_row, const TIn* __restrict__ video, int64_t vts, int64_t vqs,
                            const TIn* __restrict__ text, int64_t tts, int64_t tqs, TOut* __restrict__ packed,
                            int64_t pts, float* __restrict__ cu_out)
{
    const int chunks_per_qkv = head_row / 8;
    const int chunks_per_row = 3 * chunks_per_qkv;
    const int64_t total = (int64_t)plan.sequence_tokens * chunks_per_row;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; id < total; id += step)
    {
        const unsigned uid = (unsigned)id;  // 32-bit: the launch checks total < 2^32
        const int position = (int)(uid / (unsigned)chunks_per_row);
        const int c = (int)(uid - (unsigned)position * (unsigned)chunks_per_row);
        const int qkv = c / chunks_per_qkv;
        const int e = (c - qkv * chunks_per_qkv) * 8;
        const int source = __ldg(plan.sequence_index + position);
        const TIn* src = source < plan.source_tokens
                             ? video + (int64_t)source * vts + qkv * vqs + e
                             : text + (int64_t)(source - plan.source_tokens) * tts + qkv * tqs + e;
        float v[8];
        load8(src, v);
        store8(packed + (int64_t)position * pts + (int64_t)qkv * head_row + e, v);
    }
    if (cu_out && blockIdx.x == 0)
        for (int i = threadIdx.x; i <= plan.window_count; i += blockDim.x)
            cu_out[i] = (float)plan.cu_seqlens[i];  // cu_seqlens stored as float (awa_layers.cpp:455-456)
}

template <typename TIn, typename TOut>
__global__ void pack_scalar(PlanDevice plan, int head_row, const TIn* __restrict__ video, int64_t vts, int64_t vqs,
                            const TIn* __restrict__ text, int64_t tts, int64_t tqs, TOut* __restrict__ packed,
                            int64_t pts, float* __restrict__ cu_out)
{
    const int row = 3 * head_row;
    const int64_t total = (int64_t)plan.sequence_tokens * row;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; id < total; id += step)
    {
        const int position = (int)(id / row);
        const int c = (int)(id - (int64_t)position * row);
        const int qkv = c / head_row;
        const int e = c - qkv * head_row;
        const int source = __ldg(plan.sequence_index + position);
        const TIn* src = source < plan.source_tokens
                             ? video + (int64_t)source * vts + qkv * vqs + e
                             : text + (int64_t)(source - plan.source_tokens) * tts + qkv * tqs + e;
        store1(packed + (int64_t)position * pts + c, load1(src));
    }
    if (cu_out && blockIdx.x == 0)
        for (int i = threadIdx.x; i <= plan.window_count; i += blockDim.x)
            cu_out[i] = (float)plan.cu_seqlens[i];
}

// ---------------------------------------------------------------- MMRoPE
// Bit-exact with the reference CPU forward in fp32: each product and the
// difference/sum round separately (no FMA contraction), as the reference's
// baseline x86-64 build does.
__device__ __forceinline__ void rotate_pair(float x0, float x1, float c, float s, float& o0, float& o1)
{
    o0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    o1 = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
}

__device__ __forceinline__ float2 rope_cs(const PlanDevice& plan, short4 coords, int pair)
{
    // pair < rope_dim / 2 = 3 pairs_per_axis: the axis by two compares, not a division
    const int axis = (pair >= plan.pairs_per_axis) + (pair >= 2 * plan.pairs_per_axis);
    const int within = pair - axis * plan.pairs_per_axis;
    const int coord = axis == 0 ? coords.x : axis == 1 ? coords.y : coords.z;
    return __ldg(plan.rope_table + coord * plan.pairs_per_axis + within);
}

template <typename TIn, typename TOut>
__global__ void mmrope_chunks(PlanDevice plan, int heads, int head_dim, const TIn* __restrict__ in, int64_t its,
                              TOut* __restrict__ out, int64_t ots)
{
    const int chunks_per_row = 3 * heads * head_dim / 8;
    const int64_t total = (int64_t)plan.sequence_tokens * chunks_per_row;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    const short4* coords_table = reinterpret_cast<const short4*>(plan.position_coords);
    // e / head_dim by a multiply-high: exact while e * head_dim < 2^32 (the launch checks it)
    const uint32_t hd_magic = (uint32_t)((((uint64_t)1 << 32) + head_dim - 1) / head_dim);
    for (int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; id < total; id += step)
    {
        const unsigned uid = (unsigned)id;  // 32-bit: the launch checks total < 2^32
        const int position = (int)(uid / (unsigned)chunks_per_row);
        const int e = (int)(uid - (unsigned)position * (unsigned)chunks_per_row) * 8;
        const int qkv_head = (int)__umulhi((uint32_t)e, hd_magic);
        const int f = e - qkv_head * head_dim;
        float v[8];
        load8(in + (int64_t)position * its + e, v);
        if (qkv_head < 2 * heads && f < plan.rope_dim)
        {
            const short4 coords = coords_table[position];
#pragma unroll
            for (int i = 0; i < 4; i++)
            {
                if (f + 2 * i < plan.rope_dim)
                {
                    const float2 cs = rope_cs(plan, coords, (f >> 1) + i);
                    rotate_pair(v[2 * i], v[2 * i + 1], cs.x, cs.y, v[2 * i], v[2 * i + 1]);
                }
            }
        }
        store8(out + (int64_t)position * ots + e, v);
    }
}

template <typename TIn, typename TOut>
__global__ void mmrope_scalar(PlanDevice plan, int heads, int head_dim, const TIn* __restrict__ in, int64_t its,
                              TOut* __restrict__ out, int64_t ots)
{
    const int row = 3 * heads * head_dim;
    const int64_t total = (int64_t)plan.sequence_tokens * row;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    const short4* coords_table = reinterpret_cast<const short4*>(plan.position_coords);
    for (int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; id < total; id += step)
    {
        const int position = (int)(id / row);
        const int e = (int)(id - (int64_t)position * row);
        const int qkv_head = e / head_dim;
        const int f = e - qkv_head * head_dim;
        const TIn* src = in + (int64_t)position * its;
        float value = load1(src + e);
        if (qkv_head < 2 * heads && f < plan.rope_dim)
        {
            const float2 cs = rope_cs(plan, coords_table[position], f >> 1);
            const float paired = load1(src + (f & 1 ? e - 1 : e + 1));
            float o0, o1;
            if (f & 1)
                rotate_pair(paired, value, cs.x, cs.y, o0, o1), value = o1;
            else
                rotate_pair(value, paired, cs.x, cs.y, o0, o1), value = o0;
        }
        store1(out + (int64_t)position * ots + e, value);
    }
}

// ---------------------------------------------------------------- Unpack
template <typename TIn, typename TOut>
__global__ void unpack_video_chunks(PlanDevice plan, int head_row, const TIn* __restrict__ attended, int64_t its,
                                   TOut* __restrict__ video, int64_t vts)
{
    const int chunks_per_row = head_row / 8;
    const int64_t total = (int64_t)plan.source_tokens * chunks_per_row;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; id < total; id += step)
    {
        const int token = (int)(id / chunks_per_row);
        const int e = (int)(id - (int64_t)token * chunks_per_row) * 8;
        const int position = __ldg(plan.video_positions + token);
        float v[8];
        load8(attended + (int64_t)position * its + e, v);
        store8(video + (int64_t)token * vts + e, v);
    }
}

template <typename TIn, typename TOut>
__global__ void unpack_video_scalar(PlanDevice plan, int head_row, const TIn* __restrict__ attended, int64_t its,
                                    TOut* __restrict__ video, int64_t vts)
{
    const int64_t total = (int64_t)plan.source_tokens * head_row;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; id < total; id += step)
    {
        const int token = (int)(id / head_row);
        const int e = (int)(id - (int64_t)token * head_row);
        const int position = __ldg(plan.video_positions + token);
        store1(video + (int64_t)token * vts + e, load1(attended + (int64_t)position * its + e));
    }
}

// Text rows: out[i][e] = sum over windows (in order) of src(w, i)[e] / divisor,
// one thread per element, sequential over windows as the CPU forward
// (awa_layers.cpp:677-687), so the sum is bit-identical for identical inputs.
template <typename TIn, typename TOut>
__global__ void text_reduce(PlanDevice plan, int head_row, int packed, const TIn* __restrict__ src, int64_t sts,
                            int window_begin, int window_end, float divisor, TOut* __restrict__ out, int64_t ots)
{
    const int text = plan.text_tokens;
    const int64_t total = (int64_t)text * head_row;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; id < total; id += step)
    {
        const int i = (int)(id / head_row);
        const int e = (int)(id - (int64_t)i * head_row);
        // Eight windows' values are loaded before any is added (eight loads in
        // flight per thread); the additions stay in window order. Packed rows
        // (the Unpack layer) add x / divisor term by term, as the reference's
        // Unpack; dense partials (the fused path) are summed, then divided.
        constexpr int kBatch = 8;
        const bool term_div = packed && divisor != 0.f;
        float acc = 0.f;
        int w = window_begin;
        for (; w + kBatch <= window_end; w += kBatch)
        {
            float x[kBatch];
#pragma unroll
            for (int u = 0; u < kBatch; u++)
            {
                const int64_t row = packed ? (int64_t)__ldg(plan.cu_seqlens + w + u + 1) - text + i
                                           : (int64_t)(w + u - window_begin) * text + i;
                x[u] = load1(src + row * sts + e);
            }
#pragma unroll
            for (int u = 0; u < kBatch; u++)
                acc = __fadd_rn(acc, term_div ? __fdiv_rn(x[u], divisor) : x[u]);
        }
        for (; w < window_end; w++)
        {
            const int64_t row = packed ? (int64_t)__ldg(plan.cu_seqlens + w + 1) - text + i
                                       : (int64_t)(w - window_begin) * text + i;
            const float x = load1(src + row * sts + e);
            acc = __fadd_rn(acc, term_div ? __fdiv_rn(x, divisor) : x);
        }
        if (!packed && divisor != 0.f)
            acc = __fdiv_rn(acc, divisor);
        store1(out + (int64_t)i * ots + e, acc);
    }
}

// Two consecutive elements of a dense partial row, streamed (read once).
__device__ __forceinline__ float2 load_pair_cs(const float* p)
{
    return __ldcs(reinterpret_cast<const float2*>(p));
}

__device__ __forceinline__ float2 load_pair_cs(const __nv_bfloat16* p)
{
    const unsigned int w = __ldcs(reinterpret_cast<const unsigned int*>(p));
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// One pair of partials as loaded (raw bits), widened to fp32 when summed.
__device__ __forceinline__ float2 raw_pair_cs(const float* p) { return load_pair_cs(p); }
__device__ __forceinline__ uint32_t raw_pair_cs(const __nv_bfloat16* p)
{
    return __ldcs(reinterpret_cast<const unsigned int*>(p));
}
__device__ __forceinline__ float2 widen_pair(float2 x) { return x; }
__device__ __forceinline__ float2 widen_pair(uint32_t w)
{
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// text_reduce for dense partials ([W][text][head_row] rows of fp32 or bf16)
// whose rows and base are aligned to two elements: two consecutive elements
// per thread (more threads in flight than with 16-byte loads, which measured
// slower). Each thread's windows are a serial chain of load batches, so the
// batch is as deep as registers allow (48 bf16 or 24 fp32 pairs in flight);
// the sum in window order, then / divisor (as text_reduce does for dense
// partials).
template <typename TIn, typename TOut>
__global__ void text_reduce_v2(int text, int head_row, const TIn* __restrict__ src, int64_t sts, int windows,
                               float divisor, TOut* __restrict__ out, int64_t ots)
{
    const int pairs = head_row >> 1;
    const int64_t total = (int64_t)text * pairs;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; id < total; id += step)
    {
        const int i = (int)(id / pairs);
        const int e = (int)(id - (int64_t)i * pairs) * 2;
        const TIn* col = src + (int64_t)i * sts + e;
        const int64_t wstride = (int64_t)text * sts;  // one window's text rows
        constexpr int kBatch = sizeof(TIn) == 2 ? 48 : 24;
        float2 acc = make_float2(0.f, 0.f);
        int w = 0;
        for (; w + kBatch <= windows; w += kBatch)
        {
            decltype(raw_pair_cs(col)) x[kBatch];
#pragma unroll
            for (int u = 0; u < kBatch; u++)
                x[u] = raw_pair_cs(col + (int64_t)(w + u) * wstride);
#pragma unroll
            for (int u = 0; u < kBatch; u++)
            {
                const float2 v = widen_pair(x[u]);
                acc.x = __fadd_rn(acc.x, v.x);
                acc.y = __fadd_rn(acc.y, v.y);
            }
        }
        for (; w < windows; w++)
        {
            const float2 x = load_pair_cs(col + (int64_t)w * wstride);
            acc.x = __fadd_rn(acc.x, x.x);
            acc.y = __fadd_rn(acc.y, x.y);
        }
        if (divisor != 0.f)
        {
            acc.x = __fdiv_rn(acc.x, divisor);
            acc.y = __fdiv_rn(acc.y, divisor);
        }
        TOut* o = out + (int64_t)i * ots + e;
        store1(o, acc.x);
        store1(o + 1, acc.y);
    }
}

template <typename TOut>
__global__ void text_scale(int rows, int head_row, const float* __restrict__ sum, float divisor, TOut* __restrict__ out,
                           int64_t ots)
{
    const int64_t total = (int64_t)rows * head_row;
    for (int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; id < total; id += (int64_t)gridDim.x * blockDim.x)
    {
        const int i = (int)(id / head_row);
        const int e = (int)(id - (int64_t)i * head_row);
        store1(out + (int64_t)i * ots + e, __fdiv_rn(sum[id], divisor));
    }
}

// Video rows of windows [begin, end) between source order and the dense
// shard order (window by window, video rows only). A warp moves one token row
// (row_bytes) at a time; blockIdx.y is the window, blockIdx.x a run of
// kShardRowsPerBlock of its rows. V is the copy word: 16 bytes when row bytes,
// strides and bases are all 16-byte aligned, else 4 or 2 bytes.
constexpr int kShardRowsPerBlock = 8;

template <typename V>
__global__ void __launch_bounds__(32 * kShardRowsPerBlock)
    shard_copy_kernel(PlanDevice plan, int window_begin, int launch_begin, int row_words, const V* __restrict__ src,
                      int64_t src_stride_words, V* __restrict__ dst, int64_t dst_stride_words, int to_source)
{
    const int w = launch_begin + blockIdx.y;
    const WindowDesc win = plan.windows[w];
    const int r = blockIdx.x * kShardRowsPerBlock + (threadIdx.x >> 5);
    if (r >= win.video)
        return;
    const int64_t shard_row = (int64_t)(plan.cu_seqlens[w] - plan.cu_seqlens[window_begin]) -
                              (int64_t)(w - window_begin) * plan.text_tokens + r;
    const int plane = win.nh * win.nw;
    const int t = win.t0 + r / plane;
    const int rem = r - (r / plane) * plane;
    const int h = win.h0 + rem / win.nw;
    const int x = win.w0 + rem % win.nw;
    const int64_t token = ((int64_t)t * plan.source_h + h) * plan.source_w + x;
    const V* from = src + (to_source ? shard_row * src_stride_words : token * src_stride_words);
    V* to = dst + (to_source ? token * dst_stride_words : shard_row * dst_stride_words);
    for (int i = threadIdx.x & 31; i < row_words; i += 32)
        to[i] = from[i];
}

// fp32 QKV rows -> dense bf16 rows: a warp per token, 8 elements (32 bytes
// in, 16 out) per lane step; float4 loads when the rows are 16-byte aligned.
template <bool VEC>
__global__ void __launch_bounds__(256) rows_to_bf16_kernel(const float* __restrict__ src, int64_t ts, int64_t qs,
                                                           int tokens, int row, uint4* __restrict__ dst)
{
    const int chunks = row / 8;  // per q/k/v segment
    for (int t = blockIdx.x * 8 + (threadIdx.x >> 5); t < tokens; t += gridDim.x * 8)
        for (int c = threadIdx.x & 31; c < 3 * chunks; c += 32)
        {
            const int q = c / chunks, e = 8 * (c - q * chunks);
            const float* p = src + t * ts + q * qs + e;
            float v[8];
            if (VEC)
            {
                const float4 a = __ldg(reinterpret_cast<const float4*>(p));
                const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
                v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
            }
            else
            {
#pragma unroll
                for (int k = 0; k < 8; k++)
                    v[k] = __ldg(p + k);
            }
            uint32_t w[4];
#pragma unroll
            for (int k = 0; k < 4; k++)
            {
                const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
                w[k] = *reinterpret_cast<const uint32_t*>(&h);
            }
            dst[(int64_t)t * 3 * chunks + c] = make_uint4(w[0], w[1], w[2], w[3]);
        }
}

template <template <typename, typename> class Fn, typename... Args>
int dispatch2(int in_dtype, int out_dtype, Args&&... args)
{
    if (in_dtype == kF32 && out_dtype == kF32)
        return Fn<float, float>::run(args...);
    if (in_dtype == kF32 && out_dtype == kBF16)
        return Fn<float, bf16>::run(args...);
    if (in_dtype == kBF16 && out_dtype == kF32)
        return Fn<bf16, float>::run(args...);
    return Fn<bf16, bf16>::run(args...);
}

template <typename TIn, typename TOut>
struct PackLaunch
{
    static int run(const PlanDevice& plan, int heads, int head_dim, const void* video, int64_t vts, int64_t vqs,
                   const void* text, int64_t tts, int64_t tqs, void* packed, int64_t pts, float* cu_out,
                   cudaStream_t stream)
    {
        const int head_row = heads * head_dim;
        const void* ptrs[3] = {video, text, packed};
        const int64_t in_strides[4] = {vts, vqs, tts, tqs};
        const bool vec = chunkable(head_row, sizeof(TIn), ptrs, 2, in_strides, 4) &&
                         chunkable(head_row, sizeof(TOut), ptrs + 2, 1, &pts, 1);
        const int threads = 256;
        if (vec && (int64_t)plan.sequence_tokens * 3 * head_row / 8 < (int64_t)1 << 32)
            pack_chunks<TIn, TOut><<<grid_for((int64_t)plan.sequence_tokens * 3 * head_row / 8, threads), threads, 0,
                                     stream>>>(plan, head_row, (const TIn*)video, vts, vqs, (const TIn*)text, tts, tqs,
                                               (TOut*)packed, pts, cu_out);
        else
            pack_scalar<TIn, TOut><<<grid_for((int64_t)plan.sequence_tokens * 3 * head_row, threads), threads, 0,
                                     stream>>>(plan, head_row, (const TIn*)video, vts, vqs, (const TIn*)text, tts, tqs,
                                               (TOut*)packed, pts, cu_out);
        return (int)cudaGetLastError();
    }
};

template <typename TIn, typename TOut>
struct MmropeLaunch
{
    static int run(const PlanDevice& plan, int heads, int head_dim, const void* in, int64_t its, void* out, int64_t ots,
                   cudaStream_t stream)
    {
        const void* pin[1] = {in};
        const void* pout[1] = {out};
        const bool vec = head_dim % 8 == 0 && chunkable(3 * heads * head_dim, sizeof(TIn), pin, 1, &its, 1) &&
                         chunkable(3 * heads * head_dim, sizeof(TOut), pout, 1, &ots, 1);
        const int threads = 256;
        if (vec && (int64_t)plan.sequence_tokens * 3 * heads * head_dim / 8 < (int64_t)1 << 32 &&
            (int64_t)3 * heads * head_dim * head_dim < (int64_t)1 << 32)
            mmrope_chunks<TIn, TOut><<<grid_for((int64_t)plan.sequence_tokens * 3 * heads * head_dim / 8, threads),
                                       threads, 0, stream>>>(plan, heads, head_dim, (const TIn*)in, its, (TOut*)out, ots);
        else
            mmrope_scalar<TIn, TOut><<<grid_for((int64_t)plan.sequence_tokens * 3 * heads * head_dim, threads), threads,
                                       0, stream>>>(plan, heads, head_dim, (const TIn*)in, its, (TOut*)out, ots);
        return (int)cudaGetLastError();
    }
};

template <typename TIn, typename TOut>
struct UnpackVideoLaunch
{
    static int run(const PlanDevice& plan, int heads, int head_dim, const void* attended, int64_t its, void* video,
                   int64_t vts, cudaStream_t stream)
    {
        const int head_row = heads * head_dim;
        const void* pin[1] = {attended};
        const void* pout[1] = {video};
        const bool vec = chunkable(head_row, sizeof(TIn), pin, 1, &its, 1) &&
                         chunkable(head_row, sizeof(TOut), pout, 1, &vts, 1);
        const int threads = 256;
        if (vec)
            unpack_video_chunks<TIn, TOut><<<grid_for((int64_t)plan.source_tokens * head_row / 8, threads), threads, 0,
                                             stream>>>(plan, head_row, (const TIn*)attended, its, (TOut*)video, vts);
        else
            unpack_video_scalar<TIn, TOut><<<grid_for((int64_t)plan.source_tokens * head_row, threads), threads, 0,
                                             stream>>>(plan, head_row, (const TIn*)attended, its, (TOut*)video, vts);
        return (int)cudaGetLastError();
    }
};

// text_reduce for the Unpack layer's packed rows, two consecutive elements
// per thread: window w's text row i is packed row cu_seqlens[w + 1] - text +
// i; each term is divided by the window count before it is added, in window
// order, as the reference's Unpack does (bit-exact with text_reduce).
template <typename TIn, typename TOut>
__global__ void text_reduce_packed_v2(PlanDevice plan, int head_row, const TIn* __restrict__ src, int64_t sts,
                                      int window_begin, int window_end, float divisor, TOut* __restrict__ out,
                                      int64_t ots)
{
    const int text = plan.text_tokens;
    const int pairs = head_row >> 1;
    const int total = text * pairs;
    for (int id = blockIdx.x * blockDim.x + threadIdx.x; id < total; id += gridDim.x * blockDim.x)
    {
        const int i = id / pairs;
        const int e = (id - i * pairs) * 2;
        const TIn* col = src + (int64_t)(i - text) * sts + e;  // + cu_seqlens[w + 1] * sts
        constexpr int kBatch = sizeof(TIn) == 2 ? 32 : 16;
        float2 acc = make_float2(0.f, 0.f);
        int w = window_begin;
        for (; w + kBatch <= window_end; w += kBatch)
        {
            decltype(raw_pair_cs(col)) x[kBatch];
#pragma unroll
            for (int u = 0; u < kBatch; u++)
                x[u] = raw_pair_cs(col + (int64_t)__ldg(plan.cu_seqlens + w + u + 1) * sts);
#pragma unroll
            for (int u = 0; u < kBatch; u++)
            {
                const float2 v = widen_pair(x[u]);
                acc.x = __fadd_rn(acc.x, __fdiv_rn(v.x, divisor));
                acc.y = __fadd_rn(acc.y, __fdiv_rn(v.y, divisor));
            }
        }
        for (; w < window_end; w++)
        {
            const float2 v = load_pair_cs(col + (int64_t)__ldg(plan.cu_seqlens + w + 1) * sts);
            acc.x = __fadd_rn(acc.x, __fdiv_rn(v.x, divisor));
            acc.y = __fadd_rn(acc.y, __fdiv_rn(v.y, divisor));
        }
        TOut* o = out + (int64_t)i * ots + e;
        store1(o, acc.x);
        store1(o + 1, acc.y);
    }
}

template <typename TIn, typename TOut>
struct TextReduceLaunch
{
    static int run(const PlanDevice& plan, int heads, int head_dim, int packed, const void* src, int64_t sts,
                   int window_begin, int window_end, float divisor, void* out, int64_t ots, cudaStream_t stream)
    {
        const int head_row = heads * head_dim;
        const int threads = 256;
        if (!packed && head_row % 2 == 0 && sts % 2 == 0 && reinterpret_cast<uintptr_t>(src) % (2 * sizeof(TIn)) == 0)
        {
            const int64_t pairs = (int64_t)plan.text_tokens * (head_row / 2);
            text_reduce_v2<TIn, TOut><<<grid_for(pairs, threads), threads, 0, stream>>>(
                plan.text_tokens, head_row, (const TIn*)src, sts, window_end - window_begin, divisor, (TOut*)out,
                ots);
            return (int)cudaGetLastError();
        }
        if (packed && divisor != 0.f && head_row % 2 == 0 && sts % 2 == 0 &&
            reinterpret_cast<uintptr_t>(src) % (2 * sizeof(TIn)) == 0 && (int64_t)plan.text_tokens * head_row < (1 << 30))
        {
            const int64_t pairs = (int64_t)plan.text_tokens * (head_row / 2);
            text_reduce_packed_v2<TIn, TOut><<<grid_for(pairs, threads), threads, 0, stream>>>(
                plan, head_row, (const TIn*)src, sts, window_begin, window_end, divisor, (TOut*)out, ots);
            return (int)cudaGetLastError();
        }
        text_reduce<TIn, TOut><<<grid_for((int64_t)plan.text_tokens * head_row, threads), threads, 0, stream>>>(
            plan, head_row, packed, (const TIn*)src, sts, window_begin, window_end, divisor, (TOut*)out, ots);
        return (int)cudaGetLastError();
    }
};

}  // namespace

int launch_pack(const PlanDevice& plan, int heads, int head_dim, int in_dtype, const void* video, int64_t vts,
                int64_t vqs, const void* text, int64_t tts, int64_t tqs, int out_dtype, void* packed, int64_t pts,
                float* cu_out, cudaStream_t stream)
{
    ProfileScope prof("awa_pack", stream);
    return dispatch2<PackLaunch>(in_dtype, out_dtype, plan, heads, head_dim, video, vts, vqs, text, tts, tqs, packed,
                                 pts, cu_out, stream);
}

int launch_mmrope(const PlanDevice& plan, int heads, int head_dim, int in_dtype, const void* in, int64_t its,
                  int out_dtype, void* out, int64_t ots, cudaStream_t stream)
{
    ProfileScope prof("awa_mmrope", stream);
    return dispatch2<MmropeLaunch>(in_dtype, out_dtype, plan, heads, head_dim, in, its, out, ots, stream);
}

int launch_unpack_video(const PlanDevice& plan, int heads, int head_dim, int in_dtype, const void* attended,
                        int64_t its, int out_dtype, void* video, int64_t vts, cudaStream_t stream)
{
    ProfileScope prof("awa_unpack_video", stream);
    return dispatch2<UnpackVideoLaunch>(in_dtype, out_dtype, plan, heads, head_dim, attended, its, video, vts, stream);
}

int launch_text_reduce(const PlanDevice& plan, int heads, int head_dim, int packed, int in_dtype, const void* src,
                       int64_t src_token_stride, int window_begin, int window_end, float divisor, int out_dtype,
                       void* text_out, int64_t text_token_stride, cudaStream_t stream)
{
    ProfileScope prof("awa_text_reduce", stream);
    return dispatch2<TextReduceLaunch>(in_dtype, out_dtype, plan, heads, head_dim, packed, src, src_token_stride,
                                       window_begin, window_end, divisor, text_out, text_token_stride, stream);
}

int launch_text_scale(int rows, int heads, int head_dim, const float* text_sum, float divisor, int out_dtype,
                      void* text_out, int64_t text_token_stride, cudaStream_t stream)
{
    ProfileScope prof("awa_text_scale", stream);
    const int head_row = heads * head_dim;
    const int threads = 256;
    const int grid = grid_for((int64_t)rows * head_row, threads);
    if (out_dtype == kF32)
        text_scale<float><<<grid, threads, 0, stream>>>(rows, head_row, text_sum, divisor, (float*)text_out,
                                                        text_token_stride);
    else
        text_scale<bf16><<<grid, threads, 0, stream>>>(rows, head_row, text_sum, divisor, (bf16*)text_out,
                                                       text_token_stride);
    return (int)cudaGetLastError();
}

// Byte runs of this GPU's buffer pushed into the same offsets of peer
// buffers over NVLink (plain 16-byte loads here, 16-byte stores there):
// blockIdx.y picks the run, the threads stride through it. Every thread
// fences at system scope before it ends, so the collective the host enqueues
// next orders the stores before the peers' reads.
__global__ void __launch_bounds__(256) push_runs_kernel(const uint4* __restrict__ local, PushPeers peers,
                                                        PushRuns runs)
{
    const int r = blockIdx.y;
    const int64_t first = runs.first[r], count = runs.count[r];
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
    {
        const uint4 v = __ldg(local + first + i);
#pragma unroll 1
        for (int q = 0; q < peers.count; q++)
            peers.ptr[q][first + i] = v;
    }
    __threadfence_system();
}

int launch_rows_to_bf16(const void* src, int64_t ts, int64_t qs, int tokens, int64_t row, void* dst,
                        cudaStream_t stream)
{
    if (tokens <= 0)
        return 0;
    if (row % 8 || row > (1 << 24) || reinterpret_cast<uintptr_t>(dst) % 16)
        return (int)cudaErrorInvalidValue;
    ProfileScope prof("awa_rows_to_bf16", stream);
    const bool vec = reinterpret_cast<uintptr_t>(src) % 16 == 0 && ts % 4 == 0 && qs % 4 == 0;
    const int grid = (int)std::min<int64_t>((tokens + 7) / 8, 148 * 16);
    if (vec)
        rows_to_bf16_kernel<true><<<grid, 256, 0, stream>>>((const float*)src, ts, qs, tokens, (int)row, (uint4*)dst);
    else
        rows_to_bf16_kernel<false><<<grid, 256, 0, stream>>>((const float*)src, ts, qs, tokens, (int)row, (uint4*)dst);
    return (int)cudaGetLastError();
}

int launch_push_runs(const void* local, const PushPeers& peers, const PushRuns& runs, cudaStream_t stream)
{
    if (runs.n <= 0 || peers.count <= 0)
        return 0;
    if (runs.n > kMaxPushRuns || peers.count > kMaxPushPeers || reinterpret_cast<uintptr_t>(local) % 16)
        return (int)cudaErrorInvalidValue;
    int64_t most = 0;
    for (int r = 0; r < runs.n; r++)
        most = std::max<int64_t>(most, runs.count[r]);
    ProfileScope prof("awa_push_runs", stream);
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((most + 255) / 256, 1184 / runs.n + 1));
    push_runs_kernel<<<dim3(blocks, runs.n), 256, 0, stream>>>(static_cast<const uint4*>(local), peers, runs);
    return (int)cudaGetLastError();
}

int launch_shard_copy(const PlanDevice& plan, int heads, int head_dim, int window_begin, int window_end, int dtype,
                      const void* src, int64_t src_stride, void* dst, int64_t dst_stride, int to_source,
                      cudaStream_t stream)
{
    ProfileScope prof("awa_shard_copy", stream);
    const int64_t esize = dtype == kF32 ? 4 : 2;
    const int64_t row_bytes = (int64_t)heads * head_dim * esize;
    const int64_t sb = src_stride * esize, db = dst_stride * esize;
    // blockIdx.y is the window (at most 65535 per launch), blockIdx.x runs over
    // the longest window's video rows
    if (window_end <= window_begin)
        return 0;
    if (plan.max_window_video <= 0)
        return (int)cudaErrorInvalidValue;
    const int max_rows = plan.max_window_video;
    const dim3 block(32 * kShardRowsPerBlock);
    const uintptr_t bases = reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst);
    const bool v16 = row_bytes % 16 == 0 && sb % 16 == 0 && db % 16 == 0 && bases % 16 == 0;
    const bool v4 = row_bytes % 4 == 0 && sb % 4 == 0 && db % 4 == 0 && bases % 4 == 0;
    for (int w0 = window_begin; w0 < window_end; w0 += 65535)
    {
        // windows [w0, w1): shard rows of this launch start where window w0's do
        const int w1 = std::min(window_end, w0 + 65535);
        const dim3 grid((unsigned)((max_rows + kShardRowsPerBlock - 1) / kShardRowsPerBlock), (unsigned)(w1 - w0));
        if (v16)
            shard_copy_kernel<uint4><<<grid, block, 0, stream>>>(plan, window_begin, w0, (int)(row_bytes / 16),
                                                                 (const uint4*)src, sb / 16, (uint4*)dst, db / 16,
                                                                 to_source);
        else if (v4)
            shard_copy_kernel<uint32_t><<<grid, block, 0, stream>>>(plan, window_begin, w0, (int)(row_bytes / 4),
                                                                    (const uint32_t*)src, sb / 4, (uint32_t*)dst,
                                                                    db / 4, to_source);
        else
            shard_copy_kernel<unsigned short><<<grid, block, 0, stream>>>(
                plan, window_begin, w0, (int)(row_bytes / 2), (const unsigned short*)src, sb / 2,
                (unsigned short*)dst, db / 2, to_source);
    }
    return (int)cudaGetLastError();
}

}  // namespace awa
