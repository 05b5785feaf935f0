// awa_qkv_proj.cu -- the two GEMMs either side of the AWA layer on the tensor
// cores, x W^T with bf16 operands and fp32 accumulation in TMEM, each with its
// block's elementwise work in the epilogue:
//   kQkv  the producer of the AWA input: the QKV projection with the per-head
//         RMSNorm of Q and K (below);
//   kOut  the consumer of the AWA output: proj_out (Linear with bias), the Ada
//         "out" gate and the residual add (dit_block.py:299, 187-190, 345-347):
//         out = residual + bf16(x W^T + bias) * gate, per output channel.
//
// Math of the reference block (tools/reference/dit_block.py:280-287): the
// Linear proj_qkv (bias-free, bf16 output), then nn.RMSNorm(head_dim, eps,
// affine) on every Q and K head -- y = x * rsqrt(sum(x^2) / head_dim + eps) *
// gamma in fp32, as DitRMSNorm (src/dit/dit_precision.cpp:22-90, shader
// dit_rmsnorm.comp) computes it on the Linear's bf16 output -- and V as is.
// The output rows are the AWA layer's QKV rows: (q heads, k heads, v heads).
//
// Persistent, warp-specialised kernel, one CTA of 6 warps per SM:
//   warp 0     TMA: 64-wide K slices of x (128 token rows) and of W (256
//              output rows) into a 4-stage ring (128-byte swizzle)
//   warp 1     MMA: one lane issues 4 x tcgen05.mma (M 128, N 256, K 16) per
//              slice into one of two TMEM accumulators (256 columns each), so
//              the epilogue of a tile overlaps the MMAs of the next
//   warps 2-5  epilogue: one token row per thread; each 128-column half of
//              the tile is one head: round to bf16 (the Linear's output),
//              RMSNorm for Q and K heads, store bf16 or fp32.
// A tile is 128 tokens x 256 output features (two heads); tiles walk the
// output features fastest, so the CTAs working at the same time share their
// x rows in L2 and W (39 MB at 2560 x 7680) stays in L2.
// Every wait is bounded; a wait that gives up sets an abort flag that stops
// the other roles and reports through the device error flag.
#include "awa_internal.h"
#include "awa_rows.cuh"
#include "tcgen05.cuh"

#include <cuda.h>
#include <cuda_bf16.h>

#include <mutex>

namespace awa
{
namespace
{

using bf16 = __nv_bfloat16;

constexpr int kTileM = 128;                   // token rows per tile
constexpr int kTileN = 256;                   // output features per tile (two heads of 128)
constexpr int kTileK = 64;                    // one 128-byte swizzle row of bf16
constexpr int kStages = 4;                    // ring depth
constexpr int kATile = kTileM * kTileK * 2;   // 16 KB
constexpr int kBTile = kTileN * kTileK * 2;   // 32 KB
constexpr int kThreads = 6 * 32;
constexpr int kTmaWarp = 0, kMmaWarp = 1;  // warps 2-5: epilogue
constexpr uint32_t kTmemColumns = 2 * kTileN;  // two accumulators
constexpr uint64_t kWaitLimitNs = 4000000000ull;
constexpr uint64_t kDrainLimitNs = 200000000ull;

enum EpiMode : int
{
    kQkv = 0,
    kOut = 1
};

struct ProjArgs
{
    int tokens, model_dim, heads, n_out;  // kQkv: n_out = 3 * heads * 128
    int tiles_n, tiles, k_steps;
    const float* gamma_q;  // kQkv
    const float* gamma_k;
    float eps;
    const float* bias;  // kOut: n_out channels each
    const float* gate;
    const void* resid;  // kOut: tokens rows of n_out
    int64_t resid_stride;
    int resid_f32;
    void* out;
    int64_t out_stride;  // elements
    int out_f32;
    int* error_flag;
    // kQkv, rotated output: 0 = none, 1 = video rows (coordinates through the
    // plan's video_positions / position_coords), 2 = text rows (i, i, i)
    int rope_mode;
    PlanDevice rope;
};

struct ProjMaps
{
    CUtensorMap x, w;
};

struct ProjShared
{
    uint8_t a[kStages][kATile];
    uint8_t b[kStages][kBTile];
    uint64_t full[kStages], empty[kStages];
    uint64_t acc_full[2], acc_empty[2];
    uint64_t mma_done;
    uint32_t tmem_base;
    int abort;
};

__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort, int* error_flag, int code)
{
    if (tc::mbar_try_wait(bar, parity))
        return true;
    const uint64_t start = tc::global_ns();
    for (;;)
    {
        if (tc::mbar_try_wait_sleep(bar, parity, 20000))
            return true;
        if (*abort)
            return false;
        if (tc::global_ns() - start > kWaitLimitNs)
        {
            *abort = 1;
            if (error_flag)
                atomicCAS(error_flag, 0, code);
            return false;
        }
    }
}

__device__ __forceinline__ void drain_bar(uint64_t* bar, uint32_t parity, int* error_flag, int code)
{
    const uint64_t start = tc::global_ns();
    while (!tc::mbar_try_wait_sleep(bar, parity, 20000))
        if (tc::global_ns() - start > kDrainLimitNs)
        {
            if (error_flag)
                atomicCAS(error_flag, 0, code);
            return;
        }
}

__device__ __forceinline__ bool warp_all(bool ok)
{
    return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc::smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(tc::smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void st_v8(void* p, const uint32_t* r)
{
    asm volatile("st.global.L1::no_allocate.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}

__device__ __forceinline__ float round_bf16(float v)
{
    return __bfloat162float(__float2bfloat16_rn(v));
}

__device__ void tma_role(const ProjArgs& p, const ProjMaps& maps, ProjShared& sh)
{
    const int lane = threadIdx.x & 31;
    volatile int* abort = &sh.abort;
    uint32_t it = 0;  // K slices issued
    bool ok = true;
    for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x)
    {
        const int m0 = (t / p.tiles_n) * kTileM, n0 = (t % p.tiles_n) * kTileN;
        for (int ks = 0; ks < p.k_steps; ks++, it++)
        {
            const int stage = it % kStages;
            if (!warp_all(wait_bar(&sh.empty[stage], ((it / kStages) & 1) ^ 1, abort, p.error_flag, 61)))
            {
                ok = false;
                break;
            }
            if (lane == 0)
            {
                arrive_expect_tx(&sh.full[stage], kATile + kBTile);
                load_2d(tc::smem_addr(sh.a[stage]), &maps.x, ks * kTileK, m0, &sh.full[stage]);
                load_2d(tc::smem_addr(sh.b[stage]), &maps.w, ks * kTileK, n0, &sh.full[stage]);
            }
            __syncwarp();
        }
    }
    // the last use of each stage can still be in flight
    for (uint32_t k = 0; k < (uint32_t)kStages && k < it; k++)
    {
        const uint32_t last = it - 1 - k;
        drain_bar(&sh.full[last % kStages], (last / kStages) & 1, p.error_flag, 62);
    }
}

__device__ void mma_role(const ProjArgs& p, ProjShared& sh, uint32_t tmem)
{
    const bool leader = (threadIdx.x & 31) == 0;
    volatile int* abort = &sh.abort;
    constexpr uint32_t idesc = tc::idesc_bf16_f32(kTileM, kTileN, false);
    uint32_t it = 0;
    int i = 0;  // tiles of this CTA
    bool ok = true;
    for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x, i++)
    {
        const int buf = i & 1;
        if (!warp_all(wait_bar(&sh.acc_empty[buf], ((i >> 1) & 1) ^ 1, abort, p.error_flag, 63)))
            break;
        tc::fence_after_sync();
        const uint32_t acc = tmem + (uint32_t)(buf * kTileN);
        for (int ks = 0; ks < p.k_steps; ks++, it++)
        {
            const int stage = it % kStages;
            if (!warp_all(wait_bar(&sh.full[stage], (it / kStages) & 1, abort, p.error_flag, 64)))
            {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            if (leader)
            {
                const uint64_t a_desc = tc::smem_desc_sw128(tc::smem_addr(sh.a[stage]), 16, 1024);
                const uint64_t b_desc = tc::smem_desc_sw128(tc::smem_addr(sh.b[stage]), 16, 1024);
#pragma unroll
                for (int k = 0; k < kTileK / 16; k++)  // 32 bytes along the swizzled row per K step
                    tc::mma_ss(acc, a_desc + (uint64_t)(2 * k), b_desc + (uint64_t)(2 * k), idesc,
                               (ks | k) != 0 ? 1u : 0u);
                tc::mma_commit(&sh.empty[stage]);  // the slice's stage is free once these MMAs are done
            }
            __syncwarp();
        }
        if (!ok)
            break;
        if (leader)
            tc::mma_commit(&sh.acc_full[buf]);
        __syncwarp();
    }
    if (leader)
        tc::mma_commit(&sh.mma_done);
    __syncwarp();
    drain_bar(&sh.mma_done, 0, p.error_flag, 65);
}

// 16 consecutive residual values of a row (bf16 or fp32) into fp32.
__device__ __forceinline__ void load_resid16(const ProjArgs& p, int64_t offset, float* dst)
{
    if (p.resid_f32)
    {
        const uint4* q = reinterpret_cast<const uint4*>(static_cast<const float*>(p.resid) + offset);
#pragma unroll
        for (int u = 0; u < 4; u++)
        {
            const uint4 w = __ldg(q + u);
            dst[4 * u] = __uint_as_float(w.x);
            dst[4 * u + 1] = __uint_as_float(w.y);
            dst[4 * u + 2] = __uint_as_float(w.z);
            dst[4 * u + 3] = __uint_as_float(w.w);
        }
    }
    else
    {
        const uint4* q = reinterpret_cast<const uint4*>(static_cast<const bf16*>(p.resid) + offset);
#pragma unroll
        for (int u = 0; u < 2; u++)
        {
            const uint4 w = __ldg(q + u);
            const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int k = 0; k < 4; k++)
            {
                dst[8 * u + 2 * k] = __uint_as_float(words[k] << 16);
                dst[8 * u + 2 * k + 1] = __uint_as_float(words[k] & 0xffff0000u);
            }
        }
    }
}

// 32 values of a row into out_dtype at dst (32-byte aligned).
__device__ __forceinline__ void store32(const ProjArgs& p, char* dst, const float* v)
{
    if (p.out_f32)
    {
#pragma unroll
        for (int k = 0; k < 4; k++)
        {
            uint32_t w[8];
#pragma unroll
            for (int u = 0; u < 8; u++)
                w[u] = __float_as_uint(v[8 * k + u]);
            st_v8(dst + 32 * k, w);
        }
    }
    else
    {
#pragma unroll
        for (int k = 0; k < 2; k++)
        {
            uint32_t w[8];
#pragma unroll
            for (int u = 0; u < 8; u++)
            {
                const __nv_bfloat162 pr = __floats2bfloat162_rn(v[16 * k + 2 * u], v[16 * k + 2 * u + 1]);
                w[u] = *reinterpret_cast<const uint32_t*>(&pr);
            }
            st_v8(dst + 32 * k, w);
        }
    }
}

// kOut: out = residual + bf16(acc + bias) * gate, 32 columns at a time.
__device__ void epilogue_out(const ProjArgs& p, ProjShared& sh, uint32_t tmem)
{
    const int warp = threadIdx.x >> 5;
    const int row = (warp & 3) * 32 + (threadIdx.x & 31);  // = TMEM lane
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    volatile int* abort = &sh.abort;
    const int osz = p.out_f32 ? 4 : 2;
    int i = 0;
    for (int t = blockIdx.x; t < p.tiles; t += gridDim.x, i++)
    {
        const int buf = i & 1;
        if (!warp_all(wait_bar(&sh.acc_full[buf], (i >> 1) & 1, abort, p.error_flag, 67)))
            return;
        tc::fence_after_sync();
        const int token = (t / p.tiles_n) * kTileM + row;
        const int n0 = (t % p.tiles_n) * kTileN;
#pragma unroll 1
        for (int c = 0; c < kTileN / 32; c++)
        {
            const int f0 = n0 + 32 * c;
            uint32_t r[32];
            tc::tmem_ld32(tmem + lane_base + (uint32_t)(buf * kTileN + 32 * c), r);
            tc::tmem_wait_ld();
            if (token >= p.tokens || f0 >= p.n_out)
                continue;
            float v[32];
#pragma unroll
            for (int half = 0; half < 2; half++)
            {
                float res[16];
                load_resid16(p, (int64_t)token * p.resid_stride + f0 + 16 * half, res);
#pragma unroll
                for (int u = 0; u < 16; u++)
                {
                    const int k = 16 * half + u;
                    // bf16 Linear output (bias added first), then the two fp32
                    // roundings of hidden * gate + residual
                    v[k] = __fadd_rn(__fmul_rn(round_bf16(__uint_as_float(r[k]) + __ldg(p.bias + f0 + k)),
                                               __ldg(p.gate + f0 + k)),
                                     res[u]);
                }
            }
            store32(p, static_cast<char*>(p.out) + ((int64_t)token * p.out_stride + f0) * osz, v);
        }
        tc::fence_before_sync();
        arrive(&sh.acc_empty[buf]);
    }
}

__device__ void epilogue_qkv(const ProjArgs& p, ProjShared& sh, uint32_t tmem);

template <int MODE>
__device__ void epilogue_role(const ProjArgs& p, ProjShared& sh, uint32_t tmem)
{
    if (MODE == kOut)
        epilogue_out(p, sh, tmem);
    else
        epilogue_qkv(p, sh, tmem);
}

// kQkv: one head (128 columns) at a time: bf16 Linear output, RMSNorm of Q/K.
__device__ void epilogue_qkv(const ProjArgs& p, ProjShared& sh, uint32_t tmem)
{
    const int warp = threadIdx.x >> 5;
    const int row = (warp & 3) * 32 + (threadIdx.x & 31);  // = TMEM lane
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    volatile int* abort = &sh.abort;
    const int qk_cols = 2 * p.heads * 128;  // features of the Q and K heads
    int i = 0;
    for (int t = blockIdx.x; t < p.tiles; t += gridDim.x, i++)
    {
        const int buf = i & 1;
        const int token = (t / p.tiles_n) * kTileM + row;
        const int n0 = (t % p.tiles_n) * kTileN;
        // this row's RoPE coordinates (window-local t + text count, h, w for a
        // video token, (i, i, i) for text token i; awa_layers.cpp:896-908),
        // fetched before the wait for the accumulator
        short4 coords = make_short4(0, 0, 0, 0);
        if (p.rope_mode == 1 && token < p.tokens)
            coords = reinterpret_cast<const short4*>(p.rope.position_coords)[__ldg(p.rope.video_positions + token)];
        else if (p.rope_mode == 2)
            coords = make_short4((short)token, (short)token, (short)token, 0);
        if (!warp_all(wait_bar(&sh.acc_full[buf], (i >> 1) & 1, abort, p.error_flag, 66)))
            return;
        tc::fence_after_sync();
#pragma unroll 1
        for (int h = 0; h < 2; h++)
        {
            const int f0 = n0 + 128 * h;  // first feature of this head
            float v[128];
#pragma unroll
            for (int c = 0; c < 4; c++)
            {
                uint32_t r[32];
                tc::tmem_ld32(tmem + lane_base + (uint32_t)(buf * kTileN + 128 * h + 32 * c), r);
                tc::tmem_wait_ld();
#pragma unroll
                for (int k = 0; k < 32; k++)
                    v[32 * c + k] = __uint_as_float(r[k]);
            }
            if (token >= p.tokens || f0 >= p.n_out)
                continue;
#pragma unroll
            for (int k = 0; k < 128; k++)
                v[k] = round_bf16(v[k]);  // the Linear's bf16 output
            if (f0 < qk_cols)
            {
                // RMSNorm over the head: fp32 squares and sum (four partial sums)
                float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int k = 0; k < 128; k++)
                    s4[k & 3] = fmaf(v[k], v[k], s4[k & 3]);
                const float coef = rsqrtf(((s4[0] + s4[1]) + (s4[2] + s4[3])) / 128.f + p.eps);
                const float* gamma = f0 < qk_cols / 2 ? p.gamma_q : p.gamma_k;
#pragma unroll
                for (int k = 0; k < 128; k++)
                    v[k] = v[k] * coef * __ldg(gamma + k);
                if (p.rope_mode)
                {
                    // MMRoPE in fp32 on the normalised head, as the reference's
                    // fp32 layer (awa_layers.cpp:937-950): pair j of the first
                    // rope_dim features, axis t / h / w by pairs_per_axis
                    const int ppa = p.rope.pairs_per_axis;
#pragma unroll
                    for (int j = 0; j < 64; j++)
                    {
                        const int axis = j >= 2 * ppa ? 2 : j >= ppa ? 1 : 0;
                        const int coord = axis == 0 ? coords.x : axis == 1 ? coords.y : coords.z;
                        const bool on = 2 * j < p.rope.rope_dim;
                        const float2 cs = __ldg(p.rope.rope_table + (on ? coord * ppa + j - axis * ppa : 0));
                        float o0, o1;
                        rope_rotate(v[2 * j], v[2 * j + 1], cs.x, cs.y, o0, o1);
                        v[2 * j] = on ? o0 : v[2 * j];
                        v[2 * j + 1] = on ? o1 : v[2 * j + 1];
                    }
                }
            }
            char* dst = static_cast<char*>(p.out) + ((int64_t)token * p.out_stride + f0) * (p.out_f32 ? 4 : 2);
            if (p.out_f32)
            {
#pragma unroll
                for (int k = 0; k < 16; k++)
                {
                    uint32_t w[8];
#pragma unroll
                    for (int u = 0; u < 8; u++)
                        w[u] = __float_as_uint(v[8 * k + u]);
                    st_v8(dst + 32 * k, w);
                }
            }
            else
            {
#pragma unroll
                for (int k = 0; k < 8; k++)
                {
                    uint32_t w[8];
#pragma unroll
                    for (int u = 0; u < 8; u++)
                    {
                        const __nv_bfloat162 pr = __floats2bfloat162_rn(v[16 * k + 2 * u], v[16 * k + 2 * u + 1]);
                        w[u] = *reinterpret_cast<const uint32_t*>(&pr);
                    }
                    st_v8(dst + 32 * k, w);
                }
            }
        }
        tc::fence_before_sync();
        arrive(&sh.acc_empty[buf]);
    }
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) qkv_proj_kernel(const ProjArgs p, const __grid_constant__ ProjMaps maps)
{
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = tc::smem_addr(smem_raw);
    ProjShared& sh = *reinterpret_cast<ProjShared*>(smem_raw + ((1024 - (raw_addr & 1023)) & 1023));
    const int warp = threadIdx.x >> 5;
    if (warp == kMmaWarp)
    {
        tc::tmem_alloc(&sh.tmem_base, kTmemColumns);
        tc::tmem_relinquish();
    }
    if (threadIdx.x == 0)
    {
        for (int s = 0; s < kStages; s++)
        {
            tc::mbar_init(&sh.full[s], 1);
            tc::mbar_init(&sh.empty[s], 1);
        }
        for (int b = 0; b < 2; b++)
        {
            tc::mbar_init(&sh.acc_full[b], 1);
            tc::mbar_init(&sh.acc_empty[b], 128);
        }
        tc::mbar_init(&sh.mma_done, 1);
        tc::mbar_fence_init();
        sh.abort = 0;
    }
    if (warp == kTmaWarp && (threadIdx.x & 31) == 0)
    {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.x)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.w)) : "memory");
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = sh.tmem_base;
    if (warp == kTmaWarp)
        tma_role(p, maps, sh);
    else if (warp == kMmaWarp)
        mma_role(p, sh, tmem);
    else
        epilogue_role<MODE>(p, sh, tmem);
    tc::fence_before_sync();
    __syncthreads();
    if (warp == kMmaWarp)
    {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemColumns);
    }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult status;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &status) == cudaSuccess &&
            status == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    });
    return fn;
}

// bf16 matrix of `rows` rows of `cols` elements, `stride` elements apart; box
// of box_rows rows x 64 columns, 128-byte swizzle, zeros outside.
bool encode_matrix(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t stride, int box_rows)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn)
        return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)(stride * 2)};
    const cuuint32_t box[2] = {(cuuint32_t)kTileK, (cuuint32_t)box_rows};
    const cuuint32_t elem[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, elem,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count_proj()
{
    static int count = 0;
    if (count == 0)
    {
        int device = 0;
        cudaGetDevice(&device);
        cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device);
        if (count <= 0)
            count = 148;
    }
    return count;
}

}  // namespace

int launch_qkv_project(int tokens, int model_dim, int heads, const void* x, int64_t x_stride, const void* w,
                       int64_t w_stride, const float* gamma_q, const float* gamma_k, float eps, int out_dtype,
                       void* out, int64_t out_stride, cudaStream_t stream, const PlanDevice* rope_plan,
                       int rope_mode)
{
    const int n_out = 3 * heads * 128;
    ProjMaps maps;
    if (!encode_matrix(&maps.x, x, tokens, model_dim, x_stride, kTileM) ||
        !encode_matrix(&maps.w, w, n_out, model_dim, w_stride, kTileN))
        return (int)cudaErrorInvalidValue;
    ProjArgs p;
    p.tokens = tokens;
    p.model_dim = model_dim;
    p.heads = heads;
    p.n_out = n_out;
    p.tiles_n = (n_out + kTileN - 1) / kTileN;
    const int tiles_m = (tokens + kTileM - 1) / kTileM;
    p.tiles = tiles_m * p.tiles_n;
    p.k_steps = (model_dim + kTileK - 1) / kTileK;
    p.gamma_q = gamma_q;
    p.gamma_k = gamma_k;
    p.eps = eps;
    p.bias = p.gate = nullptr;
    p.resid = nullptr;
    p.resid_stride = 0;
    p.resid_f32 = 0;
    p.out = out;
    p.out_stride = out_stride;
    p.out_f32 = out_dtype == kF32;
    p.error_flag = device_error_flag();
    p.rope_mode = rope_plan ? rope_mode : 0;
    if (rope_plan)
        p.rope = *rope_plan;
    const size_t smem = sizeof(ProjShared) + 1024;
    cudaError_t err =
        cudaFuncSetAttribute(qkv_proj_kernel<kQkv>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess)
        return (int)err;
    ProfileScope prof(p.rope_mode ? "awa_qkv_project_rotated" : "awa_qkv_project", stream);
    const int grid = p.tiles < sm_count_proj() ? p.tiles : sm_count_proj();
    qkv_proj_kernel<kQkv><<<grid, kThreads, smem, stream>>>(p, maps);
    return (int)cudaGetLastError();
}

int launch_out_project(int tokens, int k_dim, int n_out, const void* x, int64_t x_stride, const void* w,
                       int64_t w_stride, const float* bias, const float* gate, const void* resid, int64_t resid_stride,
                       int resid_dtype, int out_dtype, void* out, int64_t out_stride, cudaStream_t stream)
{
    ProjMaps maps;
    if (!encode_matrix(&maps.x, x, tokens, k_dim, x_stride, kTileM) ||
        !encode_matrix(&maps.w, w, n_out, k_dim, w_stride, kTileN))
        return (int)cudaErrorInvalidValue;
    ProjArgs p;
    p.tokens = tokens;
    p.model_dim = k_dim;
    p.heads = 0;
    p.n_out = n_out;
    p.tiles_n = (n_out + kTileN - 1) / kTileN;
    p.tiles = ((tokens + kTileM - 1) / kTileM) * p.tiles_n;
    p.k_steps = (k_dim + kTileK - 1) / kTileK;
    p.gamma_q = p.gamma_k = nullptr;
    p.eps = 0.f;
    p.rope_mode = 0;
    p.bias = bias;
    p.gate = gate;
    p.resid = resid;
    p.resid_stride = resid_stride;
    p.resid_f32 = resid_dtype == kF32;
    p.out = out;
    p.out_stride = out_stride;
    p.out_f32 = out_dtype == kF32;
    p.error_flag = device_error_flag();
    const size_t smem = sizeof(ProjShared) + 1024;
    cudaError_t err =
        cudaFuncSetAttribute(qkv_proj_kernel<kOut>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess)
        return (int)err;
    ProfileScope prof("awa_out_project", stream);
    const int grid = p.tiles < sm_count_proj() ? p.tiles : sm_count_proj();
    qkv_proj_kernel<kOut><<<grid, kThreads, smem, stream>>>(p, maps);
    return (int)cudaGetLastError();
}

}  // namespace awa
