// awa_attn_tc.cu -- bf16 window attention on the sm_100a tensor cores
// (tcgen05.mma, fp32 accumulators in TMEM), for the bf16 DiT blocks.
//
// Math of SeedVR2WindowAttention::forward (awa_layers.cpp:1062-1120): per
// window and head, softmax(Q K^T / sqrt(d)) V over the window rows.
//
// Persistent, warp-specialised kernel: one CTA per SM walks a list of jobs;
// a job is (window, head, pair of 128-row query tiles A and B). Roles:
//
//   warps 8-11  producer. Q: each thread owns one query row (= one TMEM
//               lane), loads it from HBM into registers, rotates it (3D RoPE,
//               bf16x2 arithmetic) and writes it into TMEM with tcgen05.st --
//               Q never touches shared memory. K: 16 threads per 256-byte row,
//               global -> registers -> rotate -> 128-byte-swizzled shared
//               store. V: cp.async straight into its swizzled position.
//               K/V move through a ring of 64-key stages.
//   warp 12     MMA: one lane issues S_i = Q_i K^T (A = Q from TMEM, B = K
//               from shared memory) and O_i += P_i V (A = P from TMEM, B = V
//               read MN-major from the same swizzled layout), ping-ponging
//               between the two query tiles.
//   warps 0-3,  softmax + epilogue of tile A / tile B: each thread owns one
//   warps 4-7   query row; online max (O rescaled only when the max grows by
//               more than 2^8), exp2, P rounded to bf16 and written over S in
//               TMEM; at the end O / l is stored (video rows to source order,
//               text rows to the fp32 partials).
//
// TMEM (512 columns): Q_A 0-63, Q_B 64-127, S_A 128-191, S_B 192-255,
// O_A 256-383, O_B 384-511. Keeping Q in TMEM and rotating K on its way in
// halves the shared-memory traffic per job, which (with 128-row MMAs reading
// their B operand from shared memory) is the resource the kernel is bound by.
// Hand-offs are mbarriers (tcgen05.commit for MMA completion); every wait is
// bounded and an abort flag in shared memory stops all roles if one gives up.
#include "awa_rows.cuh"
#include "tcgen05.cuh"

#include <cuda_bf16.h>

namespace awa
{
namespace
{

using bf16 = __nv_bfloat16;

constexpr int kQRows = 128;                    // query rows per tile
constexpr int kKeys = 64;                      // keys per K/V block
constexpr int kHeadDim = 128;
constexpr int kKvPanel = kKeys * 128;          // 64 bf16 features x 64 rows (8 KB)
constexpr int kKvTile = 2 * kKvPanel;          // 64 x 128 bf16 (16 KB)
constexpr int kStages = 5;                     // K/V ring depth
constexpr int kSoftmaxWarps = 8;
constexpr int kProducerWarp0 = 8;
constexpr int kMmaWarp = 12;
constexpr int kThreads = 13 * 32;
constexpr uint32_t kTmemColumns = 512;
constexpr uint32_t kColQ = 0;    // + 64 * tile
constexpr uint32_t kColS = 128;  // + 64 * tile
constexpr uint32_t kColO = 256;  // + 128 * tile
constexpr int kRopeSmemEntries = 4096;          // (cos, sin) bf16 pairs: 16 KB
constexpr uint64_t kWaitLimitNs = 4000000000ull;  // 4 s: healthy waits last microseconds

// Source of one K/V row of a block (32 bytes, read with shared loads).
struct RowRec
{
    const void* src;  // q segment of the row for this head (nullptr: padding row)
    int64_t step;     // bytes between its q, k and v segments
    short4 coords;    // RoPE coordinates (t, h, w)
    int64_t pad;
};

struct Barriers
{
    uint64_t q_full, q_empty;
    uint64_t kv_full[kStages], kv_empty[kStages];
    uint64_t s_full[2], p_full[2], o_full[2], o_empty[2];
};

struct TcShared
{
    uint8_t kv[kStages][2][kKvTile];  // [stage][K, V]
    uint32_t rope[kRopeSmemEntries];  // the plan's bf16 (cos, sin) RoPE table
    RowRec k_rows[kKeys];
    Barriers bar;
    uint32_t tmem_base;
    int abort;
};

struct Job
{
    WindowDesc win;
    int window;
    int head;
    int qa;      // first query tile (rows 128*qa ..)
    int length;  // window rows (video + text)
    int blocks;  // 64-key blocks
    bool has_b;  // second query tile exists
};

__device__ __forceinline__ Job decode_job(const AttnArgs& a, int j)
{
    Job job;
    const int2 item = a.items[j / a.heads];
    job.head = j - (j / a.heads) * a.heads;
    job.window = item.x;
    job.win = a.plan.windows[item.x];
    job.length = job.win.video + a.plan.text_tokens;
    job.qa = 2 * item.y;
    job.blocks = (job.length + kKeys - 1) / kKeys;
    job.has_b = (job.qa + 1) * kQRows < job.length;
    return job;
}

// ---------------------------------------------------------------- waits
// Bounded mbarrier wait that also gives up when another role aborted. The
// thread sleeps inside try_wait (woken when the phase completes) and checks the
// abort flag and the time limit only when a sleep expires.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort, int* error_flag,
                                         int code)
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

__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void producer_sync()
{
    asm volatile("bar.sync 1, 128;" ::: "memory");
}

// Barrier over the 128 producer threads that also ANDs their flags, so a wait
// that gave up in one thread makes every producer thread leave together.
__device__ __forceinline__ bool producer_all(bool ok)
{
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 1, 128, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)ok)
        : "memory");
    return r != 0;
}

// Warp-uniform outcome of a bounded wait (tcgen05.ld/st are warp-collective).
__device__ __forceinline__ bool warp_all(bool ok)
{
    return __all_sync(0xffffffffu, ok);
}

// ---------------------------------------------------------------- shared-memory access
// Explicit shared-memory accesses (32-bit shared addresses), so the compiler
// knows they cannot alias global memory and keeps them in program order.
__device__ __forceinline__ void lds_row(uint32_t addr, uint64_t& src, uint64_t& step, uint64_t& coords)
{
    asm volatile("ld.shared.v2.u64 {%0, %1}, [%2];" : "=l"(src), "=l"(step) : "r"(addr));
    asm volatile("ld.shared.u64 %0, [%1+16];" : "=l"(coords) : "r"(addr));
}

__device__ __forceinline__ uint32_t lds_u32(uint32_t addr)
{
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ void sts_u4(uint32_t addr, uint4 v)
{
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w));
}

// 16-byte asynchronous global -> shared copy; src_bytes 0 writes zeros.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

__device__ __forceinline__ void cp_async_commit()
{
    asm volatile("cp.async.commit_group;" ::: "memory");
}

__device__ __forceinline__ void cp_async_wait_all()
{
    asm volatile("cp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ short4 unpack_coords(uint64_t co)
{
    return make_short4((short)(co & 0xffff), (short)((co >> 16) & 0xffff), (short)((co >> 32) & 0xffff), 0);
}

// ---------------------------------------------------------------- RoPE in bf16x2
// Rotate one bf16 pair (x0 low, x1 high) by the table entry t = (cos low, sin
// high): (x0 c - x1 s, x1 c + x0 s) = w * (c, c) + swap(w) * (-s, s).
__device__ __forceinline__ uint32_t rotate_bf16x2(uint32_t w, uint32_t t)
{
    uint32_t cc, ns, prod, sw, out;
    asm("prmt.b32 %0, %1, %1, 0x1010;" : "=r"(cc) : "r"(t));
    asm("prmt.b32 %0, %1, %1, 0x3232;" : "=r"(ns) : "r"(t));
    ns ^= 0x00008000u;  // negate the low half: (-s, s)
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(prod) : "r"(w), "r"(cc));
    asm("prmt.b32 %0, %1, %1, 0x1032;" : "=r"(sw) : "r"(w));
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(out) : "r"(sw), "r"(ns), "r"(prod));
    return out;
}

__device__ __forceinline__ int rope_axis(int pair, int ppa)
{
    return pair >= 2 * ppa ? 2 : pair >= ppa ? 1 : 0;
}

__device__ __forceinline__ int coord_of(short4 co, int axis)
{
    return axis == 0 ? co.x : axis == 1 ? co.y : co.z;
}

// Per-thread constants of the RoPE pairs of its 16-byte chunk (features 8c .. 8c+7).
struct RopeLanes
{
    int within[4];
    int axis[4];
    bool active[4];
};

__device__ __forceinline__ RopeLanes rope_lanes(const PlanDevice& plan, int c)
{
    RopeLanes rl;
#pragma unroll
    for (int i = 0; i < 4; i++)
    {
        const int pair = 4 * c + i;
        rl.active[i] = 2 * pair < plan.rope_dim;
        rl.axis[i] = rope_axis(pair, plan.pairs_per_axis);
        rl.within[i] = pair - rl.axis[i] * plan.pairs_per_axis;
    }
    return rl;
}

// ---------------------------------------------------------------- raw row loads
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
__device__ __forceinline__ uint4 to_bf16x8(const Raw8<bf16>& r)
{
    return r.u;
}
__device__ __forceinline__ uint4 to_bf16x8(const Raw8<float>& r)
{
    return make_uint4(pack_bf16x2(r.a.x, r.a.y), pack_bf16x2(r.a.z, r.a.w), pack_bf16x2(r.b.x, r.b.y),
                      pack_bf16x2(r.b.z, r.b.w));
}

// Byte offset of 16-byte chunk c (0..15 along the 128 features) of row r in a
// swizzled 64-row K/V tile: two 64-feature panels, 128-byte rows, chunk XOR row%8.
__device__ __forceinline__ uint32_t swizzled_offset(int r, int c)
{
    return (uint32_t)((c >> 3) * kKvPanel + r * 128 + ((((c & 7) ^ (r & 7))) << 4));
}

template <bool PACKED, typename TIn>
__device__ __forceinline__ void row_source(const AttnArgs& a, const Job& job, int row, const TIn*& src, int64_t& step,
                                           short4& coords)
{
    if (row < job.length)
    {
        const RowRef ref = window_row<PACKED>(a, job.win, row, job.head);
        const TIn* base =
            PACKED ? static_cast<const TIn*>(a.qkv) : static_cast<const TIn*>(ref.is_text ? a.text_qkv : a.video_qkv);
        src = base + ref.offset;
        step = ref.qkv_step;
        coords = ref.coords;
    }
    else
    {
        src = nullptr;
        step = 0;
        coords = make_short4(0, 0, 0, 0);
    }
}

// ---------------------------------------------------------------- MMA helpers
// S[128 x n] = Q K^T: A = Q from TMEM (64 columns of bf16 pairs), B = K from a
// K-major swizzled tile, 8 MMAs of K = 16 over the 128 features.
__device__ __forceinline__ void issue_qk(uint32_t tmem_s, uint32_t tmem_q, uint32_t k_addr, int n)
{
    const uint32_t idesc = tc::idesc_bf16_f32(128, n, false);
#pragma unroll
    for (int ks = 0; ks < 8; ks++)
    {
        const uint32_t off = (uint32_t)((ks >> 2) * kKvPanel + (ks & 3) * 32);
        tc::mma_ts(tmem_s, tmem_q + (uint32_t)(ks * 8), tc::smem_desc_sw128(k_addr + off, 16, 1024), idesc,
                   ks > 0 ? 1u : 0u);
    }
}

// O[128 x 128] (+)= P[128 x n] V[n x 128]; P in TMEM (bf16 pairs), V MN-major:
// 8-key groups 1024 B apart (SBO), 64-feature panels kKvPanel apart (LBO).
__device__ __forceinline__ void issue_pv(uint32_t tmem_o, uint32_t tmem_p, uint32_t v_addr, int n, bool accumulate)
{
    const uint32_t idesc = tc::idesc_bf16_f32(128, 128, true);
    for (int ks = 0; ks < n / 16; ks++)
        tc::mma_ts(tmem_o, tmem_p + (uint32_t)(ks * 8),
                   tc::smem_desc_sw128(v_addr + (uint32_t)(ks * 2048), kKvPanel, 1024), idesc,
                   (accumulate || ks > 0) ? 1u : 0u);
}

__device__ __forceinline__ int block_n(const Job& job, int kb)
{
    const int valid = min(kKeys, job.length - kb * kKeys);
    return max(16, (valid + 15) & ~15);
}

// ---------------------------------------------------------------- producer
// One query row (this thread's TMEM lane) into TMEM columns tmem_q ..+63:
// each half of the row (8 chunks) is loaded before any of it is rotated.
template <bool ROPE, typename TIn>
__device__ __forceinline__ void load_q_row(const AttnArgs& a, const TIn* src, short4 co, uint32_t tmem_q,
                                           uint32_t rope_table)
{
    const int ppa = a.plan.pairs_per_axis;
#pragma unroll
    for (int h = 0; h < 2; h++)
    {
        Raw8<TIn> raw[8];
#pragma unroll
        for (int k = 0; k < 8; k++)
        {
            if (src)
                raw[k] = load_raw(src + 8 * (8 * h + k));
            else
                zero_raw(raw[k]);
        }
        uint32_t words[32];
#pragma unroll
        for (int k = 0; k < 8; k++)
        {
            const uint4 w = to_bf16x8(raw[k]);
            words[4 * k + 0] = w.x;
            words[4 * k + 1] = w.y;
            words[4 * k + 2] = w.z;
            words[4 * k + 3] = w.w;
        }
        if (ROPE && src)
        {
#pragma unroll
            for (int k = 0; k < 32; k++)
            {
                const int pair = 32 * h + k;  // features 2 pair, 2 pair + 1
                if (2 * pair < a.plan.rope_dim)
                {
                    const int axis = rope_axis(pair, ppa);
                    const int idx = coord_of(co, axis) * ppa + pair - axis * ppa;
                    words[k] = rotate_bf16x2(words[k], lds_u32(rope_table + 4u * (uint32_t)idx));
                }
            }
        }
        tc::tmem_st32(tmem_q + (uint32_t)(32 * h), words);
    }
}

template <bool PACKED, typename TIn>
__device__ void producer_role(const AttnArgs& a, TcShared& sh, int njobs, uint32_t tmem)
{
    const int ptid = threadIdx.x - kProducerWarp0 * 32;  // = this thread's TMEM lane
    const uint32_t lane_base = (uint32_t)(ptid & ~31) << 16;
    const int c = ptid & 15;   // K/V chunk of this thread
    const int r0 = ptid >> 4;  // K/V rows r0 + 8 j
    const RopeLanes rl = rope_lanes(a.plan, c);
    const int ppa = a.plan.pairs_per_axis;
    const uint32_t rope_table = tc::smem_addr(sh.rope);
    const uint32_t k_rows = tc::smem_addr(sh.k_rows);
    volatile int* abort = &sh.abort;
    uint32_t q_empty_phase = 1;  // a fresh barrier reads as "released"
    uint32_t g = 0;              // K/V blocks produced so far
    for (int j = blockIdx.x; j < njobs; j += gridDim.x)
    {
        const Job job = decode_job(a, j);
        // ---- Q rows into TMEM (once the previous job's S MMAs are done with it)
        if (!producer_all(wait_bar(&sh.bar.q_empty, q_empty_phase, abort, a.error_flag, 11)))
            return;
        q_empty_phase ^= 1;
        tc::fence_after_sync();
#pragma unroll
        for (int t = 0; t < 2; t++)
        {
            if (t == 1 && !job.has_b)
                break;
            const TIn* src;
            int64_t step;
            short4 co;
            row_source<PACKED, TIn>(a, job, (job.qa + t) * kQRows + ptid, src, step, co);
            load_q_row<!PACKED, TIn>(a, src, co, tmem + lane_base + kColQ + 64u * t, rope_table);
        }
        tc::tmem_wait_st();
        tc::fence_before_sync();
        mbar_arrive(&sh.bar.q_full);
        // ---- K/V blocks through the ring
        for (int kb = 0; kb < job.blocks; kb++, g++)
        {
            const int stage = g % kStages;
            const uint32_t use = g / kStages;
            // also orders every producer thread after its reads of the previous row records
            if (!producer_all(wait_bar(&sh.bar.kv_empty[stage], (use & 1) ^ 1, abort, a.error_flag, 12)))
                return;
            if (ptid < kKeys)
            {
                const TIn* src;
                int64_t step;
                short4 co;
                row_source<PACKED, TIn>(a, job, kb * kKeys + ptid, src, step, co);
                RowRec& rec = sh.k_rows[ptid];
                rec.src = src;
                rec.step = step * (int64_t)sizeof(TIn);
                rec.coords = co;
            }
            producer_sync();
            const uint32_t k_tile = tc::smem_addr(sh.kv[stage][0]);
            const uint32_t v_tile = tc::smem_addr(sh.kv[stage][1]);
            uint64_t src[8], step[8], cow[8];
#pragma unroll
            for (int jj = 0; jj < 8; jj++)
                lds_row(k_rows + (uint32_t)(r0 + 8 * jj) * (uint32_t)sizeof(RowRec), src[jj], step[jj], cow[jj]);
            // V: asynchronous copies (bf16) ...
            if (sizeof(TIn) == 2)
            {
#pragma unroll
                for (int jj = 0; jj < 8; jj++)
                {
                    const char* p = src[jj] ? reinterpret_cast<const char*>(src[jj] + 2 * step[jj]) + 16 * c
                                            : reinterpret_cast<const char*>(a.plan.windows);
                    cp_async16(v_tile + swizzled_offset(r0 + 8 * jj, c), p, src[jj] ? 16u : 0u);
                }
                cp_async_commit();
            }
            // ... while K goes through registers and is rotated on the way
            // (fp32 input: V takes this path too, converted to bf16).
#pragma unroll
            for (int kv = 0; kv < (sizeof(TIn) == 2 ? 1 : 2); kv++)
            {
                Raw8<TIn> raw[8];
#pragma unroll
                for (int jj = 0; jj < 8; jj++)
                {
                    if (src[jj])
                        raw[jj] = load_raw(
                            reinterpret_cast<const TIn*>(src[jj] + (uint64_t)(1 + kv) * step[jj]) + 8 * c);
                    else
                        zero_raw(raw[jj]);
                }
#pragma unroll
                for (int jj = 0; jj < 8; jj++)
                {
                    uint4 w = to_bf16x8(raw[jj]);
                    if (!PACKED && kv == 0 && src[jj])
                    {
                        const short4 co = unpack_coords(cow[jj]);
                        uint32_t t[4];
#pragma unroll
                        for (int i = 0; i < 4; i++)
                            if (rl.active[i])
                                t[i] = lds_u32(rope_table +
                                               4u * (uint32_t)(coord_of(co, rl.axis[i]) * ppa + rl.within[i]));
                        uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                        for (int i = 0; i < 4; i++)
                            if (rl.active[i])
                                words[i] = rotate_bf16x2(words[i], t[i]);
                        w = make_uint4(words[0], words[1], words[2], words[3]);
                    }
                    sts_u4((kv == 0 ? k_tile : v_tile) + swizzled_offset(r0 + 8 * jj, c), w);
                }
            }
            if (sizeof(TIn) == 2)
                cp_async_wait_all();
            tc::fence_async_smem();
            mbar_arrive(&sh.bar.kv_full[stage]);
        }
    }
}

// ---------------------------------------------------------------- MMA issuer
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
    for (int j = blockIdx.x; j < njobs; j += gridDim.x)
    {
        const Job job = decode_job(a, j);
        const int slots = job.has_b ? 2 : 1;
        if (!warp_all(wait_bar(&sh.bar.q_full, q_full_phase, abort, a.error_flag, 21)))
            return;
        q_full_phase ^= 1;
        if (!warp_all(wait_bar(&sh.bar.kv_full[g % kStages], (g / kStages) & 1, abort, a.error_flag, 22)))
            return;
        tc::fence_after_sync();
        if (leader)
        {
            const uint32_t k_addr = tc::smem_addr(sh.kv[g % kStages][0]);
#pragma unroll
            for (int s = 0; s < 2; s++)
                if (s < slots)
                {
                    issue_qk(tmem_s[s], tmem_q[s], k_addr, block_n(job, 0));
                    tc::mma_commit(&sh.bar.s_full[s]);
                }
            if (job.blocks == 1)
                tc::mma_commit(&sh.bar.q_empty);
        }
        __syncwarp();
        for (int kb = 0; kb < job.blocks; kb++)
        {
            const uint32_t gk = g + kb;
            const int n = block_n(job, kb);
            const uint32_t v_addr = tc::smem_addr(sh.kv[gk % kStages][1]);
            const bool more = kb + 1 < job.blocks;
#pragma unroll
            for (int s = 0; s < 2; s++)
            {
                if (s >= slots)
                    break;
                if (!warp_all(wait_bar(&sh.bar.p_full[s], p_phase[s], abort, a.error_flag, 23)))
                    return;
                p_phase[s] ^= 1;
                if (kb == 0)
                {
                    if (!warp_all(wait_bar(&sh.bar.o_empty[s], o_empty_phase[s], abort, a.error_flag, 24)))
                        return;
                    o_empty_phase[s] ^= 1;
                }
                if (more && s == 0 &&
                    !warp_all(wait_bar(&sh.bar.kv_full[(gk + 1) % kStages], ((gk + 1) / kStages) & 1, abort,
                                       a.error_flag, 25)))
                    return;
                tc::fence_after_sync();
                if (leader)
                {
                    issue_pv(tmem_o[s], tmem_s[s], v_addr, n, kb > 0);
                    tc::mma_commit(&sh.bar.o_full[s]);
                    if (more)
                    {
                        // S of the next block overwrites P of this one: tcgen05.mma
                        // operations of one thread execute in issue order.
                        issue_qk(tmem_s[s], tmem_q[s], tc::smem_addr(sh.kv[(gk + 1) % kStages][0]),
                                 block_n(job, kb + 1));
                        tc::mma_commit(&sh.bar.s_full[s]);
                    }
                }
                __syncwarp();
            }
            if (leader)
            {
                if (kb + 2 == job.blocks)
                    tc::mma_commit(&sh.bar.q_empty);  // last S MMAs of the job issued: Q TMEM free when done
                tc::mma_commit(&sh.bar.kv_empty[gk % kStages]);
            }
            __syncwarp();
        }
        g += job.blocks;
    }
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
    uint32_t pv_count = 0;  // PV MMAs of this slot issued so far (o_full completions)
    for (int j = blockIdx.x; j < njobs; j += gridDim.x)
    {
        const Job job = decode_job(a, j);
        if (slot == 1 && !job.has_b)
            continue;
        const int row = (job.qa + slot) * kQRows + r;
        int64_t dst = -1;
        bool text_row = false;
        if (row < job.length)
        {
            if (PACKED)
                dst = (int64_t)(job.win.offset + row) * a.out_token_stride + (int64_t)job.head * kHeadDim;
            else if (row < job.win.video)
                dst = window_row<false>(a, job.win, row, job.head).token * a.out_token_stride +
                      (int64_t)job.head * kHeadDim;
            else
            {
                text_row = true;
                dst = ((int64_t)(job.window - a.window_begin) * text + (row - job.win.video)) * a.heads * kHeadDim +
                      (int64_t)job.head * kHeadDim;
            }
        }
        float m_run = 0.f;  // running max, in log2 units of the scaled scores
        float l_run = 0.f;
        for (int kb = 0; kb < job.blocks; kb++)
        {
            const int valid = min(kKeys, job.length - kb * kKeys);
            const bool full = valid == kKeys;
            if (!warp_all(wait_bar(&sh.bar.s_full[slot], s_phase, abort, a.error_flag, 31)))
                return;
            s_phase ^= 1;
            tc::fence_after_sync();
            uint32_t v[64];
            tc::tmem_ld32(t_s, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
            tc::tmem_ld32(t_s + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
            tc::tmem_wait_ld();
            float mxp[8];
#pragma unroll
            for (int i = 0; i < 8; i++)
                mxp[i] = -INFINITY;
#pragma unroll
            for (int i = 0; i < 64; i++)
                mxp[i & 7] = fmaxf(mxp[i & 7], (full || i < valid) ? __uint_as_float(v[i]) : -INFINITY);
            const float mx = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                                   fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
            const float m_blk = mx * scale_log2;
            float alpha = 1.f;
            bool rescale = false;
            if (kb == 0)
                m_run = m_blk;
            else if (m_blk > m_run + 8.f)
            {
                alpha = fast_exp2(m_run - m_blk);
                m_run = m_blk;
                rescale = true;
            }
            if (__any_sync(0xffffffffu, rescale))
            {
                // O of the previous block must be complete before it is scaled.
                if (!warp_all(wait_bar(&sh.bar.o_full[slot], (pv_count - 1) & 1, abort, a.error_flag, 32)))
                    return;
                tc::fence_after_sync();
#pragma unroll
                for (int cc = 0; cc < 4; cc++)
                {
                    uint32_t o[32];
                    tc::tmem_ld32(t_o + cc * 32, o);
                    tc::tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; i++)
                        o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tc::tmem_st32(t_o + cc * 32, o);
                }
            }
            // P = exp2(s * scale - max), rounded to bf16, two keys per column, over S.
            const float neg_m = -m_run;
            float sums[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int h = 0; h < 2; h++)
            {
                uint32_t pk[16];
#pragma unroll
                for (int i = 0; i < 16; i++)
                {
                    const int k = 32 * h + 2 * i;
                    const float p0 =
                        (full || k < valid) ? fast_exp2(fmaf(__uint_as_float(v[k]), scale_log2, neg_m)) : 0.f;
                    const float p1 =
                        (full || k + 1 < valid) ? fast_exp2(fmaf(__uint_as_float(v[k + 1]), scale_log2, neg_m)) : 0.f;
                    sums[i & 3] += p0 + p1;
                    pk[i] = pack_bf16x2(p0, p1);
                }
                tc::tmem_st16(t_s + 16 * h, pk);
            }
            l_run = l_run * alpha + ((sums[0] + sums[1]) + (sums[2] + sums[3]));
            tc::tmem_wait_st();
            tc::fence_before_sync();
            mbar_arrive(&sh.bar.p_full[slot]);
            pv_count++;
        }
        // epilogue: wait for the last PV, normalise, store
        if (!warp_all(wait_bar(&sh.bar.o_full[slot], (pv_count - 1) & 1, abort, a.error_flag, 33)))
            return;
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
                if (!PACKED && text_row)
                {
                    float4* out = reinterpret_cast<float4*>(a.text_partial + dst + h * 64);
#pragma unroll
                    for (int i = 0; i < 16; i++)
                        out[i] = make_float4(__uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv,
                                             __uint_as_float(o[4 * i + 2]) * inv, __uint_as_float(o[4 * i + 3]) * inv);
                }
                else if (sizeof(TOut) == 4)
                {
                    float4* out = reinterpret_cast<float4*>(static_cast<float*>(a.out) + dst + h * 64);
#pragma unroll
                    for (int i = 0; i < 16; i++)
                        out[i] = make_float4(__uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv,
                                             __uint_as_float(o[4 * i + 2]) * inv, __uint_as_float(o[4 * i + 3]) * inv);
                }
                else
                {
                    uint4* out = reinterpret_cast<uint4*>(static_cast<bf16*>(a.out) + dst + h * 64);
#pragma unroll
                    for (int i = 0; i < 8; i++)
                        out[i] = make_uint4(
                            pack_bf16x2(__uint_as_float(o[8 * i]) * inv, __uint_as_float(o[8 * i + 1]) * inv),
                            pack_bf16x2(__uint_as_float(o[8 * i + 2]) * inv, __uint_as_float(o[8 * i + 3]) * inv),
                            pack_bf16x2(__uint_as_float(o[8 * i + 4]) * inv, __uint_as_float(o[8 * i + 5]) * inv),
                            pack_bf16x2(__uint_as_float(o[8 * i + 6]) * inv, __uint_as_float(o[8 * i + 7]) * inv));
                }
            }
        }
        tc::fence_before_sync();
        mbar_arrive(&sh.bar.o_empty[slot]);
    }
}

template <bool PACKED, typename TIn, typename TOut>
__global__ void __launch_bounds__(kThreads, 1) attention_tc_kernel(const AttnArgs a)
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
        tc::mbar_init(&b.q_full, 128);
        tc::mbar_init(&b.q_empty, 1);
        for (int s = 0; s < kStages; s++)
        {
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
        tc::mbar_fence_init();
        sh.abort = 0;
    }
    // The RoPE table lives in shared memory (launch_attention_tc checks its size).
    const int rope_entries = a.plan.max_coord * a.plan.pairs_per_axis;
    for (int i = threadIdx.x; i < rope_entries; i += kThreads)
        sh.rope[i] = a.plan.rope_table_bf16[i];
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = sh.tmem_base;

    if (warp < kSoftmaxWarps)
        softmax_role<PACKED, TOut>(a, sh, njobs, tmem);
    else if (warp < kMmaWarp)
        producer_role<PACKED, TIn>(a, sh, njobs, tmem);
    else
        mma_role(a, sh, njobs, tmem);

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

template <bool PACKED, typename TIn, typename TOut>
int launch_tc(const AttnArgs& a, cudaStream_t stream)
{
    const size_t smem = sizeof(TcShared) + 1024;
    auto kernel = attention_tc_kernel<PACKED, TIn, TOut>;
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess)
        return (int)err;
    const long long jobs = (long long)a.item_count * a.heads;
    const int grid = (int)(jobs < sm_count() ? jobs : sm_count());
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
    if ((long long)args.item_count * args.heads > 0x7fffffffLL ||
        (long long)args.plan.max_coord * args.plan.pairs_per_axis > kRopeSmemEntries)
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
