// awa_attn_tc.cu -- bf16 window attention on the sm_100a tensor cores
// (tcgen05.mma, fp32 accumulators in TMEM, TMA box loads), for the bf16
// DiT blocks.
//
// Math of SeedVR2WindowAttention::forward (awa_layers.cpp:1062-1120): per
// window and head, softmax(Q K^T / sqrt(d)) V over the window rows.
//
// Persistent, warp-specialised kernel: one CTA per SM walks a list of jobs;
// a job is (window, head, pair of 128-row query tiles A and B). A window's
// rows are handled in key blocks of 64 rows:
//
//   fused path  (rows read straight from the source QKV): one block per
//               (frame, box) of the window -- a box of tc_bhc x tc_bwc tokens
//               laid over the window at its nominal (unclipped) origin, read
//               with ONE 4-D TMA load per 64 features (features x w x h x t
//               tensor map). The window rule clips windows only at the grid's
//               edges, so the part of a box outside its window lies outside
//               the grid and TMA fills it with zeros. Text rows follow in
//               blocks of 64 (2-D loads of the text QKV).
//   packed path (rows from a packed QKV, RoPE already applied): dense blocks
//               of 64 consecutive packed rows (2-D loads).
//
// Each block costs 4 TMA instructions of up to 8 KB (K and V, two 64-feature
// panels), few enough for one warp to keep HBM busy. Rows of a block that
// are not window rows (box parts outside the window, the text tail, the
// packed tail) are masked out of the softmax as keys and dropped as queries.
//
// Roles:
//   warp 13     TMA: the job's Q tiles into a staging area, K/V blocks into a
//               ring of stages (128-byte-swizzled rows, as the MMAs read them).
//   warps 8-11  RoPE: each thread owns one query row (= one TMEM lane), reads
//               it from the staging tile, rotates it (3D RoPE, bf16x2
//               arithmetic) and writes it into TMEM with tcgen05.st -- the MMA
//               reads Q from TMEM. K is rotated in place in its stage.
//   warp 12     MMA: one lane issues S_i = Q_i K^T (A = Q from TMEM, B = K
//               from shared memory) and O_i += P_i V (A = P from TMEM, B = V
//               read MN-major from the same swizzled layout), ping-ponging
//               between the two query tiles.
//   warps 0-3,  softmax + epilogue of tile A / tile B: each thread owns one
//   warps 4-7   query row; online max (O rescaled only when the max grows by
//               more than 2^8), exp2, P rounded to bf16 and written over S in
//               TMEM; at the end O / l is stored (video rows to source order,
//               text rows to the bf16 per-window partials).
//
// TMEM (512 columns): Q_A 0-63, Q_B 64-127, S_A 128-191, S_B 192-255,
// O_A 256-383, O_B 384-511. Hand-offs are mbarriers (TMA transaction counts,
// tcgen05.commit for MMA completion); every wait is bounded and an abort flag
// in shared memory stops all roles if one gives up. Before the CTA exits, the
// TMA warp waits for its copies in flight and the MMA warp for its MMAs.
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

constexpr int kQRows = 128;            // query rows per tile (two key blocks)
constexpr int kKeys = 64;              // rows per key block
constexpr int kHeadDim = 128;
constexpr int kKvPanel = kKeys * 128;  // 64 bf16 features x 64 rows (8 KB)
constexpr int kKvTile = 2 * kKvPanel;  // 64 x 128 bf16 (16 KB)
constexpr int kQPanel = kQRows * 128;  // 64 features x 128 rows (16 KB)
constexpr int kQTile = 2 * kQPanel;    // 128 x 128 bf16 (32 KB)
constexpr int kStages = 5;             // K/V ring depth (with the Q staging: 224 KB of shared memory)
constexpr int kSoftmaxWarps = 8;
constexpr int kRopeWarp0 = 8;
constexpr int kMmaWarp = 12;
constexpr int kTmaWarp = 13;
constexpr int kThreads = 14 * 32;
constexpr uint32_t kTmemColumns = 512;
constexpr uint32_t kColQ = 0;    // + 64 * tile
constexpr uint32_t kColS = 128;  // + 64 * tile
constexpr uint32_t kColO = 256;  // + 128 * tile
constexpr uint64_t kWaitLimitNs = 4000000000ull;  // 4 s: healthy waits last microseconds
constexpr uint64_t kDrainLimitNs = 200000000ull;  // 0.2 s for copies / MMAs in flight at exit
constexpr int kWaitSelftestCode = 51;                  // error code of the wait self-test

// Tensor maps of one launch, [source][q, k, v] with 128-byte swizzle and
// 64-feature boxes. Fused: source 0 = video QKV (features x w x h x t, box
// 64 x tc_bwc x tc_bhc x 1), source 1 = text QKV (features x tokens, box 64 x
// 64). Packed: source 0 = packed QKV (features x rows, box 64 x 64).
struct TmaMaps
{
    CUtensorMap map[2][3];
};

struct Barriers
{
    uint64_t q_loaded, q_free, q_full, q_empty;
    uint64_t kv_loaded[kStages], kv_full[kStages], kv_empty[kStages];
    uint64_t s_full[2], p_full[2], o_full[2], o_empty[2];
    uint64_t mma_done;
};

struct TcShared
{
    uint8_t q[2][kQTile];             // Q staging of tiles A, B
    uint8_t kv[kStages][2][kKvTile];  // [stage][K, V]
    Barriers bar;
    uint32_t tmem_base;
    int abort;
};

struct Job
{
    WindowDesc win;
    int window;
    int head;
    int qa;       // first query tile (rows 128*qa ..)
    int blocks;   // 64-row key blocks of the window
    int vblocks;  // fused: video blocks (the rest are text blocks)
    int length;   // window rows (video + text)
    bool has_b;   // second query tile exists
    bool full;    // fused: every video box lies inside the window (all 64 rows are window rows)
};

// The global-memory part of a job (its work item and window).
struct JobSource
{
    int2 item;
    WindowDesc win;
};

__device__ __forceinline__ int2 fetch_item(const AttnArgs& a, int j, int njobs)
{
    return a.items[j < njobs ? j / a.heads : 0];
}

// One stage (the softmax warps: their job starts with a wait for the first
// scores anyway, and they have no registers to spare).
__device__ __forceinline__ JobSource fetch_job(const AttnArgs& a, int j, int njobs)
{
    JobSource src;
    src.item = fetch_item(a, j, njobs);
    src.win = a.plan.windows[src.item.x];
    return src;
}

// The TMA, RoPE and MMA warps fetch job sources ahead in two stages, so that
// no load waits on another: the work item two jobs ahead and the window of
// the next job (whose item arrived a job earlier). A window load issued right
// after its item load stalls the role for a global-memory latency (about a
// microsecond) at every job boundary.
struct JobPrefetch
{
    JobSource next;  // job j + gridDim.x
    int2 item2;      // job j + 2 gridDim.x

    __device__ __forceinline__ JobPrefetch(const AttnArgs& a, int njobs)
    {
        next.item = fetch_item(a, blockIdx.x, njobs);
        next.win = a.plan.windows[next.item.x];
        item2 = fetch_item(a, blockIdx.x + gridDim.x, njobs);
    }

    // The source of job j (= the previous `next`); fetches ahead for j + gridDim.x.
    __device__ __forceinline__ JobSource advance(const AttnArgs& a, int j, int njobs)
    {
        const JobSource cur = next;
        next.item = item2;
        next.win = a.plan.windows[item2.x];
        item2 = fetch_item(a, j + 2 * gridDim.x, njobs);
        return cur;
    }
};

template <bool PACKED>
__device__ __forceinline__ Job decode_job(const AttnArgs& a, int j, const JobSource& src)
{
    Job job;
    const int2 item = src.item;
    job.head = j - (j / a.heads) * a.heads;
    job.window = item.x;
    job.win = src.win;
    job.length = job.win.video + a.plan.text_tokens;
    if (PACKED)
    {
        job.vblocks = 0;
        job.blocks = (job.length + kKeys - 1) / kKeys;
    }
    else
    {
        job.vblocks = job.win.nt * a.plan.tc_nhc * a.plan.tc_nwc;
        job.blocks = job.vblocks + a.plan.tc_text_blocks;
    }
    job.qa = 2 * item.y;
    job.has_b = 2 * (job.qa + 1) < job.blocks;
    job.full = !PACKED && job.win.h0 == job.win.h0n && job.win.w0 == job.win.w0n &&
               job.win.nh >= a.plan.tc_nhc * a.plan.tc_bhc && job.win.nw >= a.plan.tc_nwc * a.plan.tc_bwc &&
               a.plan.tc_bhc * a.plan.tc_bwc == kKeys;
    return job;
}

// Where key block b of the job comes from.
struct BlockGeo
{
    bool video;  // fused: a video box (else text rows / packed rows)
    int lt;      // video: window-local frame
    int hb, wb;  // video: box start relative to the nominal window origin
    int first;   // text: first text token; packed: first window row
};

template <bool PACKED>
__device__ __forceinline__ BlockGeo block_geo(const AttnArgs& a, const Job& job, int b)
{
    BlockGeo g;
    g.lt = g.hb = g.wb = 0;
    if (PACKED)
    {
        g.video = false;
        g.first = b * kKeys;
        return g;
    }
    g.video = b < job.vblocks;
    if (g.video)
    {
        const int per_frame = a.plan.tc_nhc * a.plan.tc_nwc;
        g.lt = b / per_frame;
        const int rem = b - g.lt * per_frame;
        const int hc = rem / a.plan.tc_nwc;
        g.hb = hc * a.plan.tc_bhc;
        g.wb = (rem - hc * a.plan.tc_nwc) * a.plan.tc_bwc;
        g.first = 0;
    }
    else
        g.first = (b - job.vblocks) * kKeys;
    return g;
}

// Walks a job's blocks in order without divisions.
struct BlockCursor
{
    int b = 0, lt = 0, hc = 0, wc = 0;

    template <bool PACKED>
    __device__ __forceinline__ BlockGeo geo(const AttnArgs& a, const Job& job) const
    {
        BlockGeo g;
        g.video = !PACKED && b < job.vblocks;
        g.lt = lt;
        g.hb = hc * a.plan.tc_bhc;
        g.wb = wc * a.plan.tc_bwc;
        g.first = PACKED ? b * kKeys : (b - job.vblocks) * kKeys;
        return g;
    }

    __device__ __forceinline__ void next(const AttnArgs& a)
    {
        b++;
        if (++wc == a.plan.tc_nwc)
        {
            wc = 0;
            if (++hc == a.plan.tc_nhc)
            {
                hc = 0;
                lt++;
            }
        }
    }
};

__device__ __forceinline__ uint64_t low_bits(int n)
{
    return n >= 64 ? ~0ull : n <= 0 ? 0ull : (1ull << n) - 1ull;
}

// Bit i set <=> row i of block b is a window row.
template <bool PACKED>
__device__ __forceinline__ uint64_t block_mask(const AttnArgs& a, const Job& job, const BlockGeo& g)
{
    if (PACKED)
        return low_bits(job.length - g.first);
    if (!g.video)
        return low_bits(a.plan.text_tokens - g.first);
    if (job.full)
        return ~0ull;
    // window part of the box: rows [h_a, h_b) x columns [w_a, w_b) of the box
    const int hoff = job.win.h0 - job.win.h0n - g.hb;
    const int woff = job.win.w0 - job.win.w0n - g.wb;
    const int h_a = max(hoff, 0), h_b = min(hoff + job.win.nh, a.plan.tc_bhc);
    const int w_a = max(woff, 0), w_b = min(woff + job.win.nw, a.plan.tc_bwc);
    if (h_a >= h_b || w_a >= w_b)
        return 0ull;
    // a box inside its window (every box of an unclipped window) covers all
    // 64 rows: skip the row loop, which every softmax and RoPE thread runs per block
    if (h_a == 0 && w_a == 0 && h_b == a.plan.tc_bhc && w_b == a.plan.tc_bwc && h_b * w_b == kKeys)
        return ~0ull;
    const uint64_t row = low_bits(w_b) & ~low_bits(w_a);
    uint64_t m = 0ull;
    for (int h = h_a; h < h_b; h++)
        m |= row << (h * a.plan.tc_bwc);
    return m;
}

// ---------------------------------------------------------------- waits
// Bounded mbarrier wait that also gives up when another role aborted. The
// thread sleeps inside try_wait (woken when the phase completes) and checks the
// abort flag and the time limit only when a sleep expires.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort, int* error_flag,
                                         int code, uint64_t limit_ns = kWaitLimitNs)
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
        if (tc::global_ns() - start > limit_ns)
        {
            *abort = 1;
            if (error_flag)
                atomicCAS(error_flag, 0, code);
            return false;
        }
    }
}

// Self-test of wait_bar: two warps wait on mbarriers that nothing completes
// (no copy, no MMA, no arrival is ever issued, so nothing is in flight when the
// block exits). Warp 0's wait has a limit of limit_ns and gives up, setting the
// abort flag and the device error flag; warp 1's wait has a limit 1000 times
// longer and must stop on the abort flag well before that. observed gets bit 0
// when warp 0 gave up, bit 1 when warp 1 stopped on the abort.
__global__ void __launch_bounds__(64) wait_selftest_kernel(uint64_t limit_ns, int* error_flag, int* observed)
{
    __shared__ uint64_t bars[2];
    __shared__ int abort_flag;
    if (threadIdx.x == 0)
    {
        tc::mbar_init(&bars[0], 1);
        tc::mbar_init(&bars[1], 1);
        abort_flag = 0;
        tc::mbar_fence_init();
    }
    __syncthreads();
    const int warp = threadIdx.x / 32;
    const uint64_t limit = warp == 0 ? limit_ns : limit_ns * 1000;
    const uint64_t start = tc::global_ns();
    const bool done = wait_bar(&bars[warp], 0, &abort_flag, warp == 0 ? error_flag : nullptr, kWaitSelftestCode, limit);
    const uint64_t took = tc::global_ns() - start;
    if ((threadIdx.x & 31) == 0 && !done)
        atomicOr(observed, warp == 0 ? 1 : (took < limit ? 2 : 0));
}

// Bounded wait used on the way out (ignores the abort flag).
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

__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc::smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(tc::smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, int w,
                                            uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(tc::smem_addr(bar))
        : "memory");
}

// One panel (64 features) of block b's rows of segment m (0 q, 1 k, 2 v)
// into shared memory at dst.
template <bool PACKED>
__device__ __forceinline__ void load_block_panel(const AttnArgs& a, const TmaMaps& maps, const Job& job,
                                                 const BlockGeo& g, int m, int panel, uint32_t dst, uint64_t* bar)
{
    const int x = job.head * kHeadDim + 64 * panel;
    if (PACKED)
        tma_load_2d(dst, &maps.map[0][m], x, job.win.offset + g.first, bar);
    else if (g.video)
        tma_load_4d(dst, &maps.map[0][m], x, job.win.w0n + g.wb, job.win.h0n + g.hb, job.win.t0 + g.lt, bar);
    else
        tma_load_2d(dst, &maps.map[1][m], x, g.first, bar);
}

// 32-byte global store (sm_100): eight 32-bit words at a 32-byte aligned address.
__device__ __forceinline__ void st_global_v8(void* p, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3, uint32_t r4,
                                             uint32_t r5, uint32_t r6, uint32_t r7)
{
    asm volatile("st.global.L1::no_allocate.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(r0), "r"(r1),
                 "r"(r2), "r"(r3), "r"(r4), "r"(r5), "r"(r6), "r"(r7)
                 : "memory");
}

// Warp-uniform outcome of a bounded wait (tcgen05.ld/st are warp-collective).
__device__ __forceinline__ bool warp_all(bool ok)
{
    return __all_sync(0xffffffffu, ok);
}

// ---------------------------------------------------------------- RoPE in bf16x2
// Rotate one bf16 pair (x0 low, x1 high) by the table entry f = ((cos, cos),
// (-sin, sin)): (x0 c - x1 s, x1 c + x0 s) = w * (c, c) + swap(w) * (-s, s).
// The table holds the two factor words ready, so a pair costs one 8-byte load
// and three instructions.
__device__ __forceinline__ uint32_t rotate_bf16x2(uint32_t w, uint2 f)
{
    const uint32_t cc = f.x, ns = f.y;
    uint32_t prod, sw, out;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(prod) : "r"(w), "r"(cc));
    asm("prmt.b32 %0, %1, %1, 0x1032;" : "=r"(sw) : "r"(w));
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(out) : "r"(sw), "r"(ns), "r"(prod));
    return out;
}

// Byte offset of 16-byte chunk c (0..15 along the 128 features) of row r in a
// swizzled tile of `rows` rows: two 64-feature panels, 128-byte rows, chunk
// XOR row%8 -- the layout the 128-byte-swizzle TMA writes from a 1024-byte
// aligned base.
__device__ __forceinline__ uint32_t swizzled_offset(int rows, int r, int c)
{
    return (uint32_t)((c >> 3) * rows * 128 + r * 128 + ((((c & 7) ^ (r & 7))) << 4));
}

// Whether the factors of `pair` and the next pair load as one 16-byte vector:
// both rotated, on one axis, the first at an even index within its axis (the
// factor rows have even length), and in the same batch of 16. Compile-time
// when RD != 0.
template <int RD>
__device__ __forceinline__ bool factors_paired(int pair, int k, int ppa, int rope_dim)
{
    const int axis = pair < ppa ? 0 : pair < 2 * ppa ? 1 : 2;
    const int q = pair - axis * ppa;
    return RD != 0 && k + 1 < 16 && (q & 1) == 0 && q + 1 < ppa && 2 * (pair + 1) < rope_dim;
}

// Rotate 32 consecutive bf16 pairs (half a 128-feature row: pairs 32*HALF ..)
// of one row whose table bases are base[x] = coord_x * stride - x * ppa (stride
// = ppa rounded up to even): the factors of pair p on axis x are at
// base[x] + p. Pairs at or past rope_dim / 2 pass through. With RD != 0, the
// axis of every pair is a compile-time constant.
template <int HALF, int RD>
__device__ __forceinline__ void rotate_half_row(uint32_t (&words)[32], const int (&base)[3], const uint2* table,
                                                int ppa_rt, int rope_dim_rt)
{
    const int ppa = RD ? RD / 6 : ppa_rt;
    const int rope_dim = RD ? RD : rope_dim_rt;
#pragma unroll
    for (int batch = 0; batch < 2; batch++)  // 16 pairs' factors (32 registers) at a time
    {
        uint2 f[16];
#pragma unroll
        for (int k = 0; k < 16; k++)
        {
            const int pair = 32 * HALF + 16 * batch + k;  // features 2 pair, 2 pair + 1
            const int b = pair < ppa ? base[0] : pair < 2 * ppa ? base[1] : base[2];
            if (k > 0 && factors_paired<RD>(pair - 1, k - 1, ppa, rope_dim))
                continue;  // loaded with the previous pair
            if (factors_paired<RD>(pair, k, ppa, rope_dim))
            {
                const uint4 v = __ldg(reinterpret_cast<const uint4*>(table + b + pair));
                f[k] = make_uint2(v.x, v.y);
                f[k + 1] = make_uint2(v.z, v.w);
            }
            else
                f[k] = __ldg(table + (2 * pair < rope_dim ? b + pair : 0));
        }
#pragma unroll
        for (int k = 0; k < 16; k++)
        {
            const int w = 16 * batch + k;
            const uint32_t rotated = rotate_bf16x2(words[w], f[k]);
            words[w] = 2 * (32 * HALF + w) < rope_dim ? rotated : words[w];
        }
    }
}

// Table bases of a window row (see rotate_half_row); zero for rows that are
// not window rows (their values are never used, any in-range entry will do).
__device__ __forceinline__ void row_bases(int (&base)[3], bool valid, const BlockGeo& geo, int text, int row_h,
                                          int row_w, int hoff, int woff, int row, int ppa)
{
    const int stride = ppa + (ppa & 1);
    int ct = 0, ch = 1, cw = 2;
    if (valid)
    {
        if (geo.video)
        {
            ct = text + geo.lt;
            ch = geo.hb + row_h - hoff;
            cw = geo.wb + row_w - woff;
        }
        else
            ct = ch = cw = geo.first + row;
    }
    base[0] = ct * stride;
    base[1] = ch * stride - ppa;
    base[2] = cw * stride - 2 * ppa;
}

__device__ __forceinline__ void load_half_row(uint32_t (&words)[32], const uint8_t* tile, int rows, int r, int half)
{
#pragma unroll
    for (int k = 0; k < 8; k++)
    {
        const uint4 w = *reinterpret_cast<const uint4*>(tile + swizzled_offset(rows, r, 8 * half + k));
        words[4 * k + 0] = w.x;
        words[4 * k + 1] = w.y;
        words[4 * k + 2] = w.z;
        words[4 * k + 3] = w.w;
    }
}

// ---------------------------------------------------------------- MMA helpers
// S[128 x n] = Q K^T: A = Q from TMEM (64 columns of bf16 pairs), B = K from a
// K-major swizzled tile, 8 MMAs of K = 16 over the 128 features.
__device__ __forceinline__ void issue_qk(uint32_t tmem_s, uint32_t tmem_q, uint32_t k_addr, int n)
{
    // The descriptor is built once; each K step only moves its start address
    // field (address >> 4): one add between MMAs keeps the issuing thread ahead
    // of the tensor core.
    const uint32_t idesc = tc::idesc_bf16_f32(128, n, false);
    const uint64_t desc = tc::smem_desc_sw128(k_addr, 16, 1024);
#pragma unroll
    for (int ks = 0; ks < 8; ks++)
    {
        constexpr uint32_t kPanelStep = kKvPanel >> 4;
        const uint64_t step = (uint64_t)((ks >> 2) * kPanelStep + (ks & 3) * 2);
        tc::mma_ts(tmem_s, tmem_q + (uint32_t)(ks * 8), desc + step, idesc, ks > 0 ? 1u : 0u);
    }
}

// O[128 x 128] (+)= P[128 x n] V[n x 128]; P in TMEM (bf16 pairs), V MN-major:
// 8-key groups 1024 B apart (SBO), 64-feature panels kKvPanel apart (LBO).
__device__ __forceinline__ void issue_pv(uint32_t tmem_o, uint32_t tmem_p, uint32_t v_addr, int n, bool accumulate)
{
    const uint32_t idesc = tc::idesc_bf16_f32(128, 128, true);
    const uint64_t desc = tc::smem_desc_sw128(v_addr, kKvPanel, 1024);
    const int steps = n / 16;
#pragma unroll
    for (int ks = 0; ks < kKeys / 16; ks++)
        if (ks < steps)
            tc::mma_ts(tmem_o, tmem_p + (uint32_t)(ks * 8), desc + (uint64_t)(ks * (2048 >> 4)), idesc,
                       (accumulate || ks > 0) ? 1u : 0u);
}

// Rows the loads of block b write: a video box writes tc_rows of the 64.
template <bool PACKED>
__device__ __forceinline__ int box_rows(const AttnArgs& a, const Job& job, int b)
{
    return (!PACKED && b < job.vblocks) ? a.plan.tc_rows : kKeys;
}

// Keys of block b that the MMAs cover (a multiple of 16): rows past them are
// never window rows. Rows below it that are not window rows are masked; they
// hold zeros or earlier rows of this launch (text rows: every window attends
// to them, so they carry nothing a window's output does not already see).
template <bool PACKED>
__device__ __forceinline__ int block_n(const AttnArgs& a, const Job& job, int b)
{
    int rows = box_rows<PACKED>(a, job, b);
    if (PACKED)
        rows = min(rows, job.length - b * kKeys);
    else if (b >= job.vblocks)
        rows = min(rows, a.plan.text_tokens - (b - job.vblocks) * kKeys);
    return max(16, (rows + 15) & ~15);
}

// ---------------------------------------------------------------- TMA warp
template <bool PACKED>
__device__ void tma_role(const AttnArgs& a, const TmaMaps& maps, TcShared& sh, int njobs)
{
    const int lane = threadIdx.x & 31;
    volatile int* abort = &sh.abort;
    uint32_t q_free_phase = 1;  // a fresh barrier reads as "released"
    uint32_t q_issued = 0;      // Q loads issued so far
    uint32_t g = 0;             // K/V blocks issued so far
    bool ok = true;
    JobPrefetch pre(a, njobs);
    for (int j = blockIdx.x; j < njobs && ok; j += gridDim.x)
    {
        const Job job = decode_job<PACKED>(a, j, pre.advance(a, j, njobs));
        // ---- the job's Q tiles (up to 4 blocks) into the staging area
        if (!warp_all(wait_bar(&sh.bar.q_free, q_free_phase, abort, a.error_flag, 41)))
            break;
        q_free_phase ^= 1;
        const int qb0 = 2 * job.qa;
        const int qblocks = min(4, job.blocks - qb0);
        if (lane == 0)
        {
            uint32_t bytes = 0;
            for (int qb = 0; qb < qblocks; qb++)
                bytes += 2u * 128u * (uint32_t)box_rows<PACKED>(a, job, qb0 + qb);
            mbar_arrive_expect_tx(&sh.bar.q_loaded, bytes);
        }
        __syncwarp();
        if (lane < 2 * qblocks)
        {
            const int qb = lane >> 1, panel = lane & 1;  // block qb0 + qb -> tile qb/2, rows 64*(qb%2)
            const uint32_t dst = tc::smem_addr(sh.q[qb >> 1]) + (uint32_t)(panel * kQPanel + (qb & 1) * kKeys * 128);
            load_block_panel<PACKED>(a, maps, job, block_geo<PACKED>(a, job, qb0 + qb), 0, panel, dst,
                                     &sh.bar.q_loaded);
        }
        q_issued++;
        // ---- K/V blocks through the ring: lanes 0-3 = (K, V) x panel
        BlockCursor cur;  // the blocks' geometry without divisions
        for (int kb = 0; kb < job.blocks; kb++, cur.next(a))
        {
            const int stage = g % kStages;
            const uint32_t use = g / kStages;
            if (!warp_all(wait_bar(&sh.bar.kv_empty[stage], (use & 1) ^ 1, abort, a.error_flag, 42)))
            {
                ok = false;
                break;
            }
            if (lane == 0)
                mbar_arrive_expect_tx(&sh.bar.kv_loaded[stage], 4u * 128u * (uint32_t)box_rows<PACKED>(a, job, kb));
            __syncwarp();
            if (lane < 4)
            {
                const int kv = lane >> 1, panel = lane & 1;
                const uint32_t dst = tc::smem_addr(sh.kv[stage][kv]) + (uint32_t)(panel * kKvPanel);
                load_block_panel<PACKED>(a, maps, job, cur.geo<PACKED>(a, job), 1 + kv, panel, dst,
                                         &sh.bar.kv_loaded[stage]);
            }
            g++;
        }
    }
    // Wait for the copies still in flight (only the last use of each barrier
    // can be outstanding: the next one is issued after the previous was consumed).
    if (q_issued > 0)
        drain_bar(&sh.bar.q_loaded, (q_issued - 1) & 1, a.error_flag, 43);
    for (uint32_t k = 0; k < (uint32_t)kStages && k < g; k++)
    {
        const uint32_t last = g - 1 - k;  // the last block issued on stage last % kStages
        drain_bar(&sh.bar.kv_loaded[last % kStages], (last / kStages) & 1, a.error_flag, 44);
    }
}

// ---------------------------------------------------------------- RoPE warps
// Every step below first issues all of its loads (data and RoPE table
// entries) and only then computes, and it never branches per pair: each pair
// is rotated and the result selected. RD is the rotated width (rope_dim) as a
// compile-time constant (126, the reference's default, with 21 pairs per
// axis), or 0 to read it from the plan; a per-pair run-time test costs the
// loop several times its arithmetic.
template <bool PACKED, int RD>
__device__ void rope_role(const AttnArgs& a, TcShared& sh, int njobs, uint32_t tmem)
{
    const int ptid = threadIdx.x - kRopeWarp0 * 32;  // = this thread's TMEM lane / Q row
    const uint32_t lane_base = (uint32_t)(ptid & ~31) << 16;
    const int kr = ptid & 63;    // K row of this thread
    const int khalf = ptid >> 6;  // ... and its half (features 64 khalf ..): warps 8-9 / 10-11
    // RD < 0: Q/K arrive rotated (by the producer's epilogue); nothing to rotate
    const int ppa = RD > 0 ? RD / 6 : a.plan.pairs_per_axis;
    const int rope_dim = RD > 0 ? RD : a.plan.rope_dim;
    const int bwc = a.plan.tc_bwc > 0 ? a.plan.tc_bwc : 1;
    const uint2* table = a.plan.rope_factors_bf16;  // read through L1
    volatile int* abort = &sh.abort;
    uint32_t q_loaded_phase = 0;
    uint32_t q_empty_phase = 1;  // TMEM Q starts free
    uint32_t g = 0;
    // (h, w) within a box of block row ptid & 63 (this thread's Q row in its
    // block, and its K row)
    const int row_h = (ptid & 63) / bwc, row_w = (ptid & 63) % bwc;

    // The job's Q tiles, rotated in place in the staging area once loaded. It
    // runs for the next job right after this job's K blocks, while the MMA warp
    // still works on this job, so that at the job boundary Q only has to be
    // copied into TMEM.
    auto prepare_q = [&](const Job& job) -> bool {
        if (!warp_all(wait_bar(&sh.bar.q_loaded, q_loaded_phase, abort, a.error_flag, 11)))
            return false;
        q_loaded_phase ^= 1;
        if (PACKED || RD < 0)
            return true;
        const int hoff = job.win.h0 - job.win.h0n, woff = job.win.w0 - job.win.w0n;
#pragma unroll 1
        for (int t = 0; t < 2; t++)
        {
            if (t == 1 && !job.has_b)
                break;
            uint8_t* tile = sh.q[t];
            int base[3];
            const int b = 2 * (job.qa + t) + (ptid >> 6);
            const BlockGeo geo = block_geo<PACKED>(a, job, b);
            const bool valid = b < job.blocks && ((block_mask<PACKED>(a, job, geo) >> (ptid & 63)) & 1ull);
            row_bases(base, valid, geo, a.plan.text_tokens, row_h, row_w, hoff, woff, ptid & 63, ppa);
            uint32_t words[32];
            load_half_row(words, tile, kQRows, ptid, 0);
            if constexpr (RD >= 0)
                rotate_half_row<0, RD>(words, base, table, ppa, rope_dim);
#pragma unroll
            for (int k = 0; k < 8; k++)
                *reinterpret_cast<uint4*>(tile + swizzled_offset(kQRows, ptid, k)) =
                    make_uint4(words[4 * k], words[4 * k + 1], words[4 * k + 2], words[4 * k + 3]);
            load_half_row(words, tile, kQRows, ptid, 1);
            if constexpr (RD >= 0)
                rotate_half_row<1, RD>(words, base, table, ppa, rope_dim);
#pragma unroll
            for (int k = 0; k < 8; k++)
                *reinterpret_cast<uint4*>(tile + swizzled_offset(kQRows, ptid, 8 + k)) =
                    make_uint4(words[4 * k], words[4 * k + 1], words[4 * k + 2], words[4 * k + 3]);
        }
        return true;
    };

    JobPrefetch pre(a, njobs);
    bool prepared = false;  // this job's Q already rotated in the staging area
    for (int j = blockIdx.x; j < njobs; j += gridDim.x)
    {
        const Job job = decode_job<PACKED>(a, j, pre.advance(a, j, njobs));
        const int hoff = job.win.h0 - job.win.h0n, woff = job.win.w0 - job.win.w0n;
        if (!prepared && !prepare_q(job))
            return;
        prepared = false;
        // ---- Q: staging (rotated) -> TMEM; tile A's row is read before the
        // wait for the TMEM columns, so that only the stores follow it
        {
            uint32_t a0[32], a1[32];
            load_half_row(a0, sh.q[0], kQRows, ptid, 0);
            load_half_row(a1, sh.q[0], kQRows, ptid, 1);
            if (!warp_all(wait_bar(&sh.bar.q_empty, q_empty_phase, abort, a.error_flag, 12)))
                return;
            q_empty_phase ^= 1;
            tc::fence_after_sync();
            tc::tmem_st32(tmem + lane_base + kColQ, a0);
            tc::tmem_st32(tmem + lane_base + kColQ + 32u, a1);
        }
        if (job.has_b)
        {
            uint32_t words[32];
            load_half_row(words, sh.q[1], kQRows, ptid, 0);
            tc::tmem_st32(tmem + lane_base + kColQ + 64u, words);
            load_half_row(words, sh.q[1], kQRows, ptid, 1);
            tc::tmem_st32(tmem + lane_base + kColQ + 96u, words);
        }
        tc::tmem_wait_st();
        tc::fence_before_sync();
        mbar_arrive(&sh.bar.q_full);
        mbar_arrive(&sh.bar.q_free);
        // ---- K blocks: rotate in place (fused); zero the V rows past the
        // window's end (packed: they belong to the next window); hand the
        // stage to the MMA
        BlockCursor cur;
        for (int kb = 0; kb < job.blocks; kb++, g++, cur.next(a))
        {
            const int stage = g % kStages;
            const uint32_t use = g / kStages;
            const BlockGeo geo = cur.geo<PACKED>(a, job);
            const uint64_t mask = block_mask<PACKED>(a, job, geo);
            if (!warp_all(wait_bar(&sh.bar.kv_loaded[stage], use & 1, abort, a.error_flag, 13)))
                return;
            if constexpr (!PACKED && RD < 0)
            {
                // K arrived rotated: the stage goes to the MMA as loaded
            }
            else if (!PACKED)
            {
                // one row, half its features, per thread (same shape as the Q step)
                uint8_t* k_tile = sh.kv[stage][0];
                int base[3];
                row_bases(base, (mask >> kr) & 1ull, geo, a.plan.text_tokens, row_h, row_w, hoff, woff, kr, ppa);
                uint32_t words[32];
                load_half_row(words, k_tile, kKeys, kr, khalf);
                if constexpr (RD >= 0)
                {
                    if (khalf == 0)
                        rotate_half_row<0, RD>(words, base, table, ppa, rope_dim);
                    else
                        rotate_half_row<1, RD>(words, base, table, ppa, rope_dim);
                }
#pragma unroll
                for (int k = 0; k < 8; k++)
                    *reinterpret_cast<uint4*>(k_tile + swizzled_offset(kKeys, kr, 8 * khalf + k)) =
                        make_uint4(words[4 * k], words[4 * k + 1], words[4 * k + 2], words[4 * k + 3]);
                // generic-proxy writes -> visible to the tensor core's async-proxy reads
                tc::fence_async_smem();
            }
            else if (mask != ~0ull)
            {
                uint8_t* v_tile = sh.kv[stage][1];
                if (!((mask >> kr) & 1ull))
                {
#pragma unroll
                    for (int k = 0; k < 8; k++)
                        *reinterpret_cast<uint4*>(v_tile + swizzled_offset(kKeys, kr, 8 * khalf + k)) =
                            make_uint4(0, 0, 0, 0);
                }
                tc::fence_async_smem();
            }
            mbar_arrive(&sh.bar.kv_full[stage]);
        }
        if (j + (int)gridDim.x < njobs)
        {
            if (!prepare_q(decode_job<PACKED>(a, j + gridDim.x, pre.next)))
                return;
            prepared = true;
        }
    }
}

// ---------------------------------------------------------------- MMA issuer
template <bool PACKED>
__device__ void mma_role(const AttnArgs& a, TcShared& sh, int njobs, uint32_t tmem)
{
    const bool leader = (threadIdx.x & 31) == 0;
    volatile int* abort = &sh.abort;
    uint32_t q_full_phase = 0;
    uint32_t p_phase[2] = {0, 0};
    uint32_t o_empty_phase[2] = {1, 1};
    uint32_t g = 0;  // K/V blocks consumed so far
    const uint32_t tmem_q[2] = {tmem + kColQ, tmem + kColQ + 64};
    const uint32_t tmem_s[2] = {tmem + kColS, tmem + kColS + 64};
    const uint32_t tmem_o[2] = {tmem + kColO, tmem + kColO + 128};
    bool ok = true;
    JobPrefetch pre(a, njobs);
    for (int j = blockIdx.x; j < njobs && ok; j += gridDim.x)
    {
        const Job job = decode_job<PACKED>(a, j, pre.advance(a, j, njobs));
        const int slots = job.has_b ? 2 : 1;
        if (!warp_all(wait_bar(&sh.bar.q_full, q_full_phase, abort, a.error_flag, 21)))
            break;
        q_full_phase ^= 1;
        if (!warp_all(wait_bar(&sh.bar.kv_full[g % kStages], (g / kStages) & 1, abort, a.error_flag, 22)))
            break;
        tc::fence_after_sync();
        if (leader)
        {
            const uint32_t k_addr = tc::smem_addr(sh.kv[g % kStages][0]);
#pragma unroll
            for (int s = 0; s < 2; s++)
                if (s < slots)
                {
                    issue_qk(tmem_s[s], tmem_q[s], k_addr, block_n<PACKED>(a, job, 0));
                    tc::mma_commit(&sh.bar.s_full[s]);
                }
            if (job.blocks == 1)
                tc::mma_commit(&sh.bar.q_empty);
        }
        __syncwarp();
        for (int kb = 0; kb < job.blocks && ok; kb++)
        {
            const uint32_t gk = g + kb;
            const int n = block_n<PACKED>(a, job, kb);
            const uint32_t v_addr = tc::smem_addr(sh.kv[gk % kStages][1]);
            const bool more = kb + 1 < job.blocks;
#pragma unroll
            for (int s = 0; s < 2; s++)
            {
                if (s >= slots)
                    break;
                if (!warp_all(wait_bar(&sh.bar.p_full[s], p_phase[s], abort, a.error_flag, 23)))
                {
                    ok = false;
                    break;
                }
                p_phase[s] ^= 1;
                if (kb == 0)
                {
                    if (!warp_all(wait_bar(&sh.bar.o_empty[s], o_empty_phase[s], abort, a.error_flag, 24)))
                    {
                        ok = false;
                        break;
                    }
                    o_empty_phase[s] ^= 1;
                }
                if (more && s == 0 &&
                    !warp_all(wait_bar(&sh.bar.kv_full[(gk + 1) % kStages], ((gk + 1) / kStages) & 1, abort,
                                       a.error_flag, 25)))
                {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                if (leader)
                {
                    issue_pv(tmem_o[s], tmem_s[s], v_addr, n, kb > 0);
                    if (more)
                    {
                        // S of the next block overwrites P of this one: tcgen05.mma
                        // operations of one thread execute in issue order. The
                        // commit covers this P V too (a commit tracks every MMA the
                        // thread issued before it): the softmax may scale O once
                        // the next scores are in.
                        issue_qk(tmem_s[s], tmem_q[s], tc::smem_addr(sh.kv[(gk + 1) % kStages][0]),
                                 block_n<PACKED>(a, job, kb + 1));
                        tc::mma_commit(&sh.bar.s_full[s]);
                    }
                    else
                        tc::mma_commit(&sh.bar.o_full[s]);  // the job's O is complete
                }
                __syncwarp();
            }
            if (!ok)
                break;
            if (leader)
            {
                if (kb + 2 == job.blocks)
                    tc::mma_commit(&sh.bar.q_empty);  // last S MMAs of the job issued: Q TMEM free when done
                // (the stage of this block is released by the softmax warps of
                // the job's last slot, which see every MMA that read it complete)
            }
            __syncwarp();
        }
        g += job.blocks;
    }
    // every MMA this thread issued is complete before TMEM is released
    if (leader)
        tc::mma_commit(&sh.bar.mma_done);
    __syncwarp();
    drain_bar(&sh.bar.mma_done, 0, a.error_flag, 26);
}

// ---------------------------------------------------------------- packed fp32 helpers
// sm_100 executes two fp32 lanes per instruction for add / mul / fma on
// register pairs (.f32x2) and takes three operands in max.f32: the softmax's
// arithmetic is bound by the FMA-pipe issue it shares with the RoPE warps, so
// it uses those forms. Each lane rounds as the scalar instruction does.
__device__ __forceinline__ void fma_x2(float& d0, float& d1, float a0, float a1, float b, float c)
{
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %4};\n\t"
        "mov.b64 rc, {%5, %5};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b), "f"(c));
}

__device__ __forceinline__ void add_x2(float& acc0, float& acc1, float a0, float a1)
{
    asm("{\n\t.reg .b64 ra, rb;\n\t"
        "mov.b64 ra, {%0, %1};\n\t"
        "mov.b64 rb, {%2, %3};\n\t"
        "add.rn.f32x2 ra, ra, rb;\n\t"
        "mov.b64 {%0, %1}, ra;\n\t}"
        : "+f"(acc0), "+f"(acc1)
        : "f"(a0), "f"(a1));
}

__device__ __forceinline__ void mul_x2(float& d0, float& d1, float a0, float a1, float b)
{
    asm("{\n\t.reg .b64 ra, rb;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %4};\n\t"
        "mul.rn.f32x2 ra, ra, rb;\n\t"
        "mov.b64 {%0, %1}, ra;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b));
}

__device__ __forceinline__ float max3(float a, float b, float c)
{
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// ---------------------------------------------------------------- softmax + epilogue
template <bool PACKED, typename TOut>
__device__ void softmax_role(const AttnArgs& a, TcShared& sh, int njobs, uint32_t tmem)
{
    const int warp = threadIdx.x >> 5;
    const int slot = warp >> 2;
    const int r = threadIdx.x & 127;  // query row within the tile = TMEM lane
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem + kColS + (uint32_t)(slot * 64) + lane_base;
    const uint32_t t_o = tmem + kColO + (uint32_t)(slot * 128) + lane_base;
    const float scale_log2 = a.scale * 1.4426950408889634f;
    const int text = a.plan.text_tokens;
    volatile int* abort = &sh.abort;
    uint32_t s_phase = 0;
    uint32_t o_phase = 0;   // o_full completes once per job of this slot
    uint32_t g = 0;         // K/V blocks of the jobs before this one
    JobSource next = fetch_job(a, blockIdx.x, njobs);
    for (int j = blockIdx.x; j < njobs; j += gridDim.x)
    {
        const Job job = decode_job<PACKED>(a, j, next);
        next = fetch_job(a, j + gridDim.x, njobs);
        g += job.blocks;
        if (slot == 1 && !job.has_b)
            continue;
        // The slot whose MMAs the MMA warp issues last in each block (B if the
        // job has it) hands the ring stages back to the TMA warp: its commit
        // after the next block's scores covers every MMA that read this block.
        // One thread of it arrives; g - blocks is the job's first ring entry.
        const bool releases = slot == (int)job.has_b && r == 0;
        // this thread's query row: row i of block qb
        const int qb = 2 * (job.qa + slot) + (r >> 6);
        const int qi = r & 63;
        int64_t dst = -1;
        bool text_row = false;
        if (qb < job.blocks)
        {
            const BlockGeo geo = block_geo<PACKED>(a, job, qb);
            if ((block_mask<PACKED>(a, job, geo) >> qi) & 1ull)
            {
                if (PACKED)
                    dst = (int64_t)(job.win.offset + geo.first + qi) * a.out_token_stride +
                          (int64_t)job.head * kHeadDim;
                else if (geo.video)
                {
                    const int h = job.win.h0n + geo.hb + qi / a.plan.tc_bwc;
                    const int w = job.win.w0n + geo.wb + qi % a.plan.tc_bwc;
                    const int64_t token =
                        ((int64_t)(job.win.t0 + geo.lt) * a.plan.source_h + h) * a.plan.source_w + w;
                    dst = token * a.out_token_stride + (int64_t)job.head * kHeadDim;
                }
                else
                {
                    text_row = true;
                    const int slot = a.partial_slot ? a.partial_slot[job.window] : job.window - a.window_begin;
                    dst = ((int64_t)slot * text + (geo.first + qi)) * a.heads * kHeadDim + (int64_t)job.head * kHeadDim;
                }
            }
        }
        float m_run = -INFINITY;  // running max, in log2 units of the scaled scores
        float l_run = 0.f;
        BlockCursor cur;
        for (int kb = 0; kb < job.blocks; kb++, cur.next(a))
        {
            const uint64_t mask = block_mask<PACKED>(a, job, cur.geo<PACKED>(a, job));
            if (!warp_all(wait_bar(&sh.bar.s_full[slot], s_phase, abort, a.error_flag, 31)))
                return;
            s_phase ^= 1;
            tc::fence_after_sync();
            if (releases && kb > 0)
                mbar_arrive(&sh.bar.kv_empty[(g - job.blocks + kb - 1) % kStages]);
            uint32_t v[64];
            tc::tmem_ld32(t_s, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
            tc::tmem_ld32(t_s + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
            tc::tmem_wait_ld();
            if (mask != ~0ull)
            {
#pragma unroll
                for (int i = 0; i < 64; i++)
                    if (!((mask >> i) & 1ull))
                        v[i] = 0xff800000u;  // -inf: p = 0
            }
            float mxp[4];
#pragma unroll
            for (int i = 0; i < 4; i++)
                mxp[i] = -INFINITY;
#pragma unroll
            for (int i = 0; i < 32; i++)
                mxp[i & 3] = max3(mxp[i & 3], __uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
            const float mx = max3(max3(mxp[0], mxp[1], mxp[2]), mxp[3], -INFINITY);
            const float m_blk = mx * scale_log2;
            float alpha = 1.f;
            bool rescale = false;
            if (kb == 0)
                m_run = m_blk;
            else if (m_blk > m_run + 8.f)
            {
                alpha = fast_exp2(m_run - m_blk);  // 0 while no key has been seen (m_run = -inf)
                m_run = m_blk;
                rescale = true;
            }
            if (__any_sync(0xffffffffu, rescale))
            {
                // O holds P V of the blocks before this one, complete: the MMA warp
                // committed these scores after issuing the previous block's P V.
                // 16 columns at a time: the 64 scores stay in registers meanwhile
#pragma unroll 1
                for (int cc = 0; cc < 8; cc++)
                {
                    uint32_t o[16];
                    tc::tmem_ld16(t_o + cc * 16, o);
                    tc::tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 16; i += 2)
                    {
                        float a0, a1;
                        mul_x2(a0, a1, __uint_as_float(o[i]), __uint_as_float(o[i + 1]), alpha);
                        o[i] = __float_as_uint(a0);
                        o[i + 1] = __float_as_uint(a1);
                    }
                    tc::tmem_st16(t_o + cc * 16, o);
                }
            }
            // P = exp2(s * scale - max), rounded to bf16, two keys per column, over S.
            // (No key seen yet: m_run = -inf and every p is 0.)
            const float neg_m = m_run == -INFINITY ? 0.f : -m_run;
            float sums[4] = {0.f, 0.f, 0.f, 0.f};  // two lane pairs
#pragma unroll
            for (int h = 0; h < 2; h++)
            {
                uint32_t pk[16];
#pragma unroll
                for (int i = 0; i < 16; i++)
                {
                    const int k = 32 * h + 2 * i;
                    float x0, x1;
                    fma_x2(x0, x1, __uint_as_float(v[k]), __uint_as_float(v[k + 1]), scale_log2, neg_m);
                    const float p0 = fast_exp2(x0);
                    const float p1 = fast_exp2(x1);
                    add_x2(sums[2 * (i & 1)], sums[2 * (i & 1) + 1], p0, p1);
                    pk[i] = pack_bf16x2(p0, p1);
                }
                tc::tmem_st16(t_s + 16 * h, pk);
            }
            l_run = l_run * alpha + ((sums[0] + sums[1]) + (sums[2] + sums[3]));
            tc::tmem_wait_st();
            tc::fence_before_sync();
            mbar_arrive(&sh.bar.p_full[slot]);
        }
        // epilogue: wait for the last PV, normalise, store
        if (!warp_all(wait_bar(&sh.bar.o_full[slot], o_phase, abort, a.error_flag, 33)))
            return;
        o_phase ^= 1;
        if (releases)
            mbar_arrive(&sh.bar.kv_empty[(g - 1) % kStages]);
        tc::fence_after_sync();
        const float inv = 1.f / l_run;
#pragma unroll
        for (int h = 0; h < 2; h++)
        {
            uint32_t o[64];
            tc::tmem_ld32(t_o + h * 64, *reinterpret_cast<uint32_t(*)[32]>(&o[0]));
            tc::tmem_ld32(t_o + h * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&o[32]));
            tc::tmem_wait_ld();
            if (dst >= 0)
            {
                // this thread's row: 64 fp32 (fp32 out) or bf16 values (bf16 out, and
                // the text partials, as the layer chain's bf16 attended rows)
                const bool f32 = !(!PACKED && text_row) && sizeof(TOut) == 4;
                char* row = (!PACKED && text_row)
                                ? reinterpret_cast<char*>(reinterpret_cast<bf16*>(a.text_partial) + dst + h * 64)
                                : static_cast<char*>(a.out) + (dst + h * 64) * (int64_t)sizeof(TOut);
                if (f32)
                {
#pragma unroll
                    for (int i = 0; i < 64; i += 2)
                    {
                        float a0, a1;
                        mul_x2(a0, a1, __uint_as_float(o[i]), __uint_as_float(o[i + 1]), inv);
                        o[i] = __float_as_uint(a0);
                        o[i + 1] = __float_as_uint(a1);
                    }
                    if (a.out_v8)
                    {
#pragma unroll
                        for (int i = 0; i < 8; i++)
                            st_global_v8(row + 32 * i, o[8 * i], o[8 * i + 1], o[8 * i + 2], o[8 * i + 3], o[8 * i + 4],
                                         o[8 * i + 5], o[8 * i + 6], o[8 * i + 7]);
                    }
                    else
                    {
#pragma unroll
                        for (int i = 0; i < 16; i++)
                            reinterpret_cast<uint4*>(row)[i] = make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
                    }
                }
                else
                {
                    uint32_t pk[32];
#pragma unroll
                    for (int i = 0; i < 32; i++)
                    {
                        float a0, a1;
                        mul_x2(a0, a1, __uint_as_float(o[2 * i]), __uint_as_float(o[2 * i + 1]), inv);
                        pk[i] = pack_bf16x2(a0, a1);
                    }
                    if (a.out_v8)
                    {
#pragma unroll
                        for (int i = 0; i < 4; i++)
                            st_global_v8(row + 32 * i, pk[8 * i], pk[8 * i + 1], pk[8 * i + 2], pk[8 * i + 3],
                                         pk[8 * i + 4], pk[8 * i + 5], pk[8 * i + 6], pk[8 * i + 7]);
                    }
                    else
                    {
#pragma unroll
                        for (int i = 0; i < 8; i++)
                            reinterpret_cast<uint4*>(row)[i] =
                                make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
                    }
                }
            }
        }
        tc::fence_before_sync();
        mbar_arrive(&sh.bar.o_empty[slot]);
    }
}

template <bool PACKED, typename TOut, int RD>
__global__ void __launch_bounds__(kThreads, 1)
    attention_tc_kernel(const AttnArgs a, const __grid_constant__ TmaMaps maps)
{
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the 128-byte swizzle atoms.
    const uint32_t raw_addr = tc::smem_addr(smem_raw);
    TcShared& sh = *reinterpret_cast<TcShared*>(smem_raw + ((1024 - (raw_addr & 1023)) & 1023));
    const int warp = threadIdx.x >> 5;
    const int njobs = a.item_count * a.heads;

    if (warp == kMmaWarp)
    {
        tc::tmem_alloc(&sh.tmem_base, kTmemColumns);
        tc::tmem_relinquish();
    }
    if (threadIdx.x == 0)
    {
        Barriers& b = sh.bar;
        tc::mbar_init(&b.q_loaded, 1);
        tc::mbar_init(&b.q_free, 128);
        tc::mbar_init(&b.q_full, 128);
        tc::mbar_init(&b.q_empty, 1);
        for (int s = 0; s < kStages; s++)
        {
            tc::mbar_init(&b.kv_loaded[s], 1);
            tc::mbar_init(&b.kv_full[s], 128);
            tc::mbar_init(&b.kv_empty[s], 1);
        }
        for (int s = 0; s < 2; s++)
        {
            tc::mbar_init(&b.s_full[s], 1);
            tc::mbar_init(&b.p_full[s], 128);
            tc::mbar_init(&b.o_full[s], 1);
            tc::mbar_init(&b.o_empty[s], 128);
        }
        tc::mbar_init(&b.mma_done, 1);
        tc::mbar_fence_init();
        sh.abort = 0;
    }
    if (warp == kTmaWarp && (threadIdx.x & 31) == 0)
    {
        for (int s = 0; s < 2; s++)
            for (int m = 0; m < 3; m++)
                asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.map[s][m]))
                             : "memory");
    }
    // Start from zeros: rows that no load of this launch writes stay zero.
    {
        uint4* z = reinterpret_cast<uint4*>(&sh.q[0][0]);
        const int n = (int)((sizeof(sh.q) + sizeof(sh.kv)) / sizeof(uint4));
        for (int i = threadIdx.x; i < n; i += kThreads)
            z[i] = make_uint4(0, 0, 0, 0);
    }
    tc::fence_async_smem();  // the zeros land before any TMA write or MMA read
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = sh.tmem_base;

    if (warp < kSoftmaxWarps)
        softmax_role<PACKED, TOut>(a, sh, njobs, tmem);
    else if (warp < kMmaWarp)
        rope_role<PACKED, RD>(a, sh, njobs, tmem);
    else if (warp == kMmaWarp)
        mma_role<PACKED>(a, sh, njobs, tmem);
    else
        tma_role<PACKED>(a, maps, sh, njobs);

    tc::fence_before_sync();
    __syncthreads();
    if (warp == kMmaWarp)
    {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemColumns);
    }
}

int sm_count()
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

// ---------------------------------------------------------------- tensor maps (host)
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled()
{
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult status;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &status) == cudaSuccess &&
            status == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// bf16 tensor map of `rank` dims (dim 0 = features, contiguous), strides in
// bytes for dims 1.., box dims, 128-byte swizzle, zero fill outside.
bool encode(CUtensorMap* map, const void* base, int rank, const int64_t* dims, const int64_t* strides,
            const int* box)
{
    EncodeTiledFn fn = encode_tiled();
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15))
        return false;
    cuuint64_t d[4], s[3];
    cuuint32_t b[4], e[4];
    for (int i = 0; i < rank; i++)
    {
        if (dims[i] <= 0 || box[i] <= 0 || box[i] > 256)
            return false;
        d[i] = (cuuint64_t)dims[i];
        b[i] = (cuuint32_t)box[i];
        e[i] = 1;
        if (i > 0)
        {
            if (strides[i - 1] % 16 || strides[i - 1] <= 0)
                return false;
            s[i - 1] = (cuuint64_t)strides[i - 1];
        }
    }
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank, const_cast<void*>(base), d, s, b, e,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool build_maps(const AttnArgs& a, int packed, TmaMaps& maps)
{
    const PlanDevice& p = a.plan;
    const int64_t row = (int64_t)a.heads * a.head_dim;
    for (int m = 0; m < 3; m++)
    {
        if (packed)
        {
            const char* base = static_cast<const char*>(a.qkv) + (int64_t)m * row * 2;
            const int64_t dims[2] = {row, p.sequence_tokens};
            const int64_t strides[1] = {a.qkv_token_stride * 2};
            const int box[2] = {64, kKeys};
            if (!encode(&maps.map[0][m], base, 2, dims, strides, box))
                return false;
            maps.map[1][m] = maps.map[0][m];
            continue;
        }
        const char* vbase = static_cast<const char*>(a.video_qkv) + (int64_t)m * a.video_qkv_stride * 2;
        const int64_t t_stride = a.video_token_stride * 2;
        const int64_t vdims[4] = {row, p.source_w, p.source_h, p.source_t};
        const int64_t vstrides[3] = {t_stride, t_stride * p.source_w, t_stride * p.source_w * p.source_h};
        const int vbox[4] = {64, p.tc_bwc, p.tc_bhc, 1};
        if (!encode(&maps.map[0][m], vbase, 4, vdims, vstrides, vbox))
            return false;
        const char* tbase = static_cast<const char*>(a.text_qkv) + (int64_t)m * a.text_qkv_stride * 2;
        const int64_t tdims[2] = {row, p.text_tokens};
        const int64_t tstrides[1] = {a.text_token_stride * 2};
        const int tbox[2] = {64, kKeys};
        if (!encode(&maps.map[1][m], tbase, 2, tdims, tstrides, tbox))
            return false;
    }
    return true;
}

template <bool PACKED, typename TOut, int RD>
int launch_tc(const AttnArgs& a, const TmaMaps& maps, cudaStream_t stream)
{
    const size_t smem = sizeof(TcShared) + 1024;
    auto kernel = attention_tc_kernel<PACKED, TOut, RD>;
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess)
        return (int)err;
    const long long jobs = (long long)a.item_count * a.heads;
    const int grid = (int)(jobs < sm_count() ? jobs : sm_count());
    kernel<<<grid, kThreads, smem, stream>>>(a, maps);
    return (int)cudaGetLastError();
}

}  // namespace

int launch_wait_selftest(uint64_t limit_ns, int* error_flag, int* observed, cudaStream_t stream)
{
    wait_selftest_kernel<<<1, 64, 0, stream>>>(limit_ns, error_flag, observed);
    return (int)cudaGetLastError();
}

int launch_attention_tc(const AttnArgs& args, int packed, int in_dtype, int out_dtype, cudaStream_t stream)
{
    const PlanDevice& p = args.plan;
    if (args.head_dim != kHeadDim || in_dtype != kBF16)
        return (int)cudaErrorInvalidValue;
    if ((long long)args.item_count * args.heads > 0x7fffffffLL ||
        p.tc_rows <= 0 || p.tc_rows > kKeys ||
        p.text_tokens <= 0)
        return (int)cudaErrorInvalidValue;
    TmaMaps maps;
    if (!build_maps(args, packed, maps))
        return (int)cudaErrorInvalidValue;
    AttnArgs a = args;
    const int64_t out_size = out_dtype == kF32 ? 4 : 2;
    a.out_v8 = (reinterpret_cast<uintptr_t>(args.out) % 32 == 0) && (args.out_token_stride * out_size) % 32 == 0 &&
               (reinterpret_cast<uintptr_t>(args.text_partial) % 32 == 0) && (args.heads * args.head_dim * 2) % 32 == 0;
    ProfileScope prof(packed ? "awa_attention_tc_packed"
                             : args.rotate ? "awa_attention_tc_fused" : "awa_attention_tc_prerotated",
                      stream);
    // The packed path applies no RoPE; the fused path has a 126-wide (21 pairs per axis) instance.
    const bool rd126 = p.rope_dim == 126 && p.pairs_per_axis == 21;
    // Q/K rotated by the producer: the instance without rotation (RD = -1)
    const bool rotated = !packed && !args.rotate;
    if (out_dtype == kF32)
    {
        if (packed)
            return launch_tc<true, float, 0>(a, maps, stream);
        if (rotated)
            return launch_tc<false, float, -1>(a, maps, stream);
        return rd126 ? launch_tc<false, float, 126>(a, maps, stream) : launch_tc<false, float, 0>(a, maps, stream);
    }
    if (packed)
        return launch_tc<true, bf16, 0>(a, maps, stream);
    if (rotated)
        return launch_tc<false, bf16, -1>(a, maps, stream);
    return rd126 ? launch_tc<false, bf16, 126>(a, maps, stream) : launch_tc<false, bf16, 0>(a, maps, stream);
}

}  // namespace awa
