// awa_shard.cpp -- one AWA layer split over the GPUs of a node
// (include/awa_b200.h: awa_comm_*, awa_shard_*, awa_forward_sharded).
//
// Windows are independent (SeedVR2WindowAttention::forward runs each window on
// its own, awa_layers.cpp:1062-1120); the only coupling between them is the
// text mean text[i] = sum_w attended_text(w)[i] / W (awa_layers.cpp:684-685).
// So each rank computes a share of the layer and the ranks exchange the rest:
//
//   window split: the windows sharing a (t-range, h-range) form a band
//     (frames x whole grid lines); bands in (t, h) order are cut into one run
//     of near-equal cost per rank, so a rank's video rows are a few contiguous
//     token runs. The fp32 text partial sums are NCCL all-reduced. The video
//     runs go to every rank's output: pushed straight into the other ranks'
//     copies when video_out lies in a buffer shared over the ranks
//     (awa_comm_alloc_shared: CUDA IPC), by the copy engines behind the
//     attention or by an SM push kernel after it; else packed, NCCL
//     all-gathered and copied back into place;
//   head split (few bands or windows): rank r runs the whole layer for a range
//     of heads -- the QKV and output pointers offset by the first head, the
//     row strides unchanged -- and the head slices are exchanged.
//
// Every rank ends with the full video and text outputs, as the ncnn boundary
// requires. No attention kernel touches a peer's memory and nothing uses TMA
// multicast; libnccl.so.2 is opened at run time, so the library loads on
// machines without NCCL, and inside a PyTorch process the dynamic loader hands
// back the NCCL that torch already loaded.
#include "awa_b200.h"
#include "awa_internal.h"

#include <dlfcn.h>

#include <nccl.h>

#include <algorithm>
#include <array>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <type_traits>
#include <vector>

#include <cuda_runtime.h>

namespace
{

// ---------------------------------------------------------------- NCCL entry points
struct Nccl
{
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_count)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*comm_user_rank)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
};

const Nccl* nccl()
{
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h)
            h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h)
            return;
        auto sym = [h](auto& fn, const char* name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            return fn != nullptr;
        };
        n.ok = sym(n.get_unique_id, "ncclGetUniqueId") && sym(n.comm_init_rank, "ncclCommInitRank") &&
               sym(n.comm_destroy, "ncclCommDestroy") && sym(n.comm_count, "ncclCommCount") &&
               sym(n.comm_user_rank, "ncclCommUserRank") && sym(n.all_gather, "ncclAllGather") &&
               sym(n.all_reduce, "ncclAllReduce") && sym(n.group_start, "ncclGroupStart") &&
               sym(n.group_end, "ncclGroupEnd") && sym(n.error_string, "ncclGetErrorString");
    });
    return n.ok ? &n : nullptr;
}

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...)
{
    char message[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(message, sizeof(message), fmt, ap);
    va_end(ap);
    return awa::report_error(code, message);
}

int nccl_status(const Nccl* n, ncclResult_t r, const char* what)
{
    if (r == ncclSuccess)
        return AWA_OK;
    return fail(AWA_ERR_CUDA, "%s: %s", what, n->error_string(r));
}

int cuda_status(cudaError_t e, const char* what)
{
    if (e == cudaSuccess)
        return AWA_OK;
    return fail(AWA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

size_t align256(size_t v)
{
    return (v + 255) & ~(size_t)255;
}

size_t dsize(int dtype)
{
    return dtype == AWA_BF16 ? 2 : 4;
}

}  // namespace

// A device buffer of every rank mapped into every rank's address space (CUDA
// IPC): peer[q] is rank q's buffer (peer[rank] the local one).
struct SharedBuffer
{
    void* local = nullptr;
    size_t bytes = 0;
    std::vector<void*> peer;
};

struct awa_comm
{
    ncclComm_t comm = nullptr;
    int rank = 0;
    int nranks = 1;
    int device = -1;
    bool owned = false;
    std::vector<SharedBuffer> shared;
    int* barrier_word = nullptr;  // device int for the entry barrier of the direct mode
    // direct mode: the peer copies of video rows, one stream per peer (copies
    // to different peers run on different copy engines at once), the events
    // that start a chunk's copies and those that join them back
    std::vector<cudaStream_t> push_stream;
    cudaEvent_t chunk_ready[8] = {};
    std::vector<cudaEvent_t> push_done;
    int push_mode = AWA_PUSH_AUTO;  // how direct mode moves the video rows
};

namespace
{

// How one layer is split over the ranks of a communicator.
//
// Window split: the windows tile the grid as a product of t-, h- and
// w-intervals, so the windows sharing a (t-interval, h-interval) form a band:
// frames [t0, t1) x grid lines [h0, h1) x every column. Bands in (t, h) order
// are cut into nranks runs of near-equal attention cost (sum of L^2 over the
// band's windows). A rank then owns whole grid lines: per frame of each of
// its bands one contiguous run of tokens, merged across frames where a band
// spans every line -- so its video rows leave it in a few large copies.
struct Band
{
    int t0, t1, h0, h1;
    double cost;               // sum of L^2 over its windows
    std::vector<int> windows;  // plan indices, ascending
};

struct Split
{
    bool by_heads = false;
    std::vector<int> bounds;  // head split: head bounds; window split: windows before each rank (prefix sums)
    std::vector<Band> bands;  // window split: in (t, h) order
    std::vector<std::vector<int>> rank_bands;  // per rank: its bands, in order
    std::vector<std::vector<int>> windows;     // per rank: its windows, ascending
    int64_t slot_rows = 0;                     // most video rows of one rank
};

// The windows of some bands, ascending.
std::vector<int> band_windows(const Split& s, const int* bands, int n)
{
    std::vector<int> w;
    for (int i = 0; i < n; i++)
        w.insert(w.end(), s.bands[bands[i]].windows.begin(), s.bands[bands[i]].windows.end());
    std::sort(w.begin(), w.end());
    return w;
}

// The token runs (first token, tokens) of some bands in token order: every
// (frame, line range) of the bands, sorted, adjacent ones merged -- so the
// bands of one frame slab that cover all its lines become a single run.
std::vector<std::pair<int64_t, int64_t>> band_runs(const Split& s, const awa_plan_info& info, const int* bands, int n)
{
    std::vector<std::pair<int64_t, int64_t>> pieces;
    const int64_t line = info.source_w;
    for (int i = 0; i < n; i++)
    {
        const Band& b = s.bands[bands[i]];
        for (int t = b.t0; t < b.t1; t++)
            pieces.emplace_back(((int64_t)t * info.source_h + b.h0) * line, (int64_t)(b.h1 - b.h0) * line);
    }
    std::sort(pieces.begin(), pieces.end());
    std::vector<std::pair<int64_t, int64_t>> runs;
    for (const auto& p : pieces)
        if (!runs.empty() && runs.back().first + runs.back().second == p.first)
            runs.back().second += p.second;
        else
            runs.push_back(p);
    return runs;
}

Split make_split(const awa_plan* plan, const awa_plan_info& info, int nranks, int heads)
{
    Split s;
    s.bounds.assign(nranks + 1, 0);
    std::vector<awa_window> win(info.window_count);
    awa_plan_get_maps(plan, nullptr, nullptr, nullptr, nullptr, win.data());
    {
        std::map<std::array<int, 4>, size_t> index;
        for (int w = 0; w < info.window_count; w++)
        {
            const awa_window& x = win[w];
            const std::array<int, 4> key{x.t0, x.h0, x.t1, x.h1};
            auto it = index.find(key);
            if (it == index.end())
            {
                it = index.emplace(key, s.bands.size()).first;
                s.bands.push_back(Band{x.t0, x.t1, x.h0, x.h1, 0.0, {}});
            }
            Band& b = s.bands[it->second];
            const double L = (double)(x.t1 - x.t0) * (x.h1 - x.h0) * (x.w1 - x.w0) + info.text_tokens;
            b.cost += L * L;
            b.windows.push_back(w);
        }
        std::sort(s.bands.begin(), s.bands.end(),
                  [](const Band& a, const Band& b) { return a.t0 != b.t0 ? a.t0 < b.t0 : a.h0 < b.h0; });
    }
    s.by_heads = nranks > 1 && heads >= nranks && ((int)s.bands.size() < nranks || info.window_count < 4 * nranks);
    if (s.by_heads)
    {
        for (int r = 0; r <= nranks; r++)
            s.bounds[r] = (int)((int64_t)heads * r / nranks);
        return s;
    }
    // bands -> ranks in order: each band goes to the rank whose equal share of
    // the total cost its cost midpoint falls in
    double total = 0;
    for (const Band& b : s.bands)
        total += b.cost;
    s.rank_bands.assign(nranks, {});
    double acc = 0;
    for (size_t i = 0; i < s.bands.size(); i++)
    {
        const double mid = acc + 0.5 * s.bands[i].cost;
        s.rank_bands[std::min(nranks - 1, (int)(mid / total * nranks))].push_back((int)i);
        acc += s.bands[i].cost;
    }
    s.windows.resize(nranks);
    for (int r = 0; r < nranks; r++)
    {
        const auto& rb = s.rank_bands[r];
        s.windows[r] = band_windows(s, rb.data(), (int)rb.size());
        int64_t rows = 0;
        for (const auto& run : band_runs(s, info, rb.data(), (int)rb.size()))
            rows += run.second;
        s.slot_rows = std::max(s.slot_rows, rows);
        s.bounds[r + 1] = s.bounds[r] + (int)s.windows[r].size();
    }
    return s;
}

// Workspace layout of awa_forward_sharded (offsets in bytes, each 256-aligned).
struct Layout
{
    size_t text_sum = 0, forward = 0, gather = 0, text_gather = 0, total = 0;
};

Layout make_layout(const awa_plan* plan, const awa_plan_info& info, const Split& s, int nranks, int heads,
                   int head_dim, int out_dtype)
{
    Layout l;
    const size_t row = (size_t)heads * head_dim;
    size_t off = 0;
    l.text_sum = off;
    off += align256((size_t)info.text_tokens * row * sizeof(float));
    l.forward = off;
    if (s.by_heads)
    {
        int most = 0;
        for (int r = 0; r < nranks; r++)
            most = std::max(most, s.bounds[r + 1] - s.bounds[r]);
        off += align256(awa_forward_workspace_bytes(plan, most, head_dim));
        l.gather = off;
        // slots of [N_v][most heads][d] video rows, then [T][most heads][d] text rows
        off += align256((size_t)nranks * info.source_tokens * most * head_dim * dsize(out_dtype));
        l.text_gather = off;
        off += align256((size_t)nranks * info.text_tokens * most * head_dim * dsize(out_dtype));
    }
    else
    {
        size_t most = 1;
        for (const auto& w : s.windows)
            most = std::max(most, w.size());
        off += align256(most * info.text_tokens * row * sizeof(float));
        l.gather = off;
        off += align256((size_t)nranks * std::max<int64_t>(s.slot_rows, 1) * row * dsize(out_dtype));
        l.text_gather = off;
    }
    l.total = off;
    return l;
}

// The shared buffer that holds [p, p + bytes) on this rank, or nullptr.
const SharedBuffer* find_shared(const awa_comm* c, const void* p, size_t bytes)
{
    const unsigned char* q = static_cast<const unsigned char*>(p);
    for (const SharedBuffer& b : c->shared)
    {
        const unsigned char* base = static_cast<const unsigned char*>(b.local);
        if (q >= base && q + bytes <= base + b.bytes)
            return &b;
    }
    return nullptr;
}

void release_shared(SharedBuffer& b, int rank)
{
    for (size_t q = 0; q < b.peer.size(); q++)
        if ((int)q != rank && b.peer[q])
            cudaIpcCloseMemHandle(b.peer[q]);
    if (b.local)
        cudaFree(b.local);
    b = SharedBuffer();
}

// All ranks reach this point on `stream` before any goes on (a one-word NCCL
// all-reduce).
int barrier(const Nccl* n, awa_comm* c, cudaStream_t stream)
{
    return nccl_status(n, n->all_reduce(c->barrier_word, c->barrier_word, 1, ncclInt32, ncclSum, c->comm, stream),
                       "ncclAllReduce (barrier)");
}

// ---------------------------------------------------------------- direct mode pushes
constexpr int kPushChunks = 3;  // attention launches per rank, each followed by its rows' peer copies

// The peer-copy streams and events (made once per communicator).
int push_streams(awa_comm* c)
{
    if (!c->push_stream.empty())
        return AWA_OK;
    cudaError_t e = cudaSuccess;
    for (int q = 0; q < c->nranks - 1 && e == cudaSuccess; q++)
    {
        cudaStream_t s = nullptr;
        cudaEvent_t d = nullptr;
        e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
        if (e == cudaSuccess)
            e = cudaEventCreateWithFlags(&d, cudaEventDisableTiming);
        c->push_stream.push_back(s);
        c->push_done.push_back(d);
    }
    for (int i = 0; i < kPushChunks && e == cudaSuccess; i++)
        e = cudaEventCreateWithFlags(&c->chunk_ready[i], cudaEventDisableTiming);
    return cuda_status(e, "peer copy streams");
}

// The rank's bands cut into at most kPushChunks runs: returns the band-list
// offsets of the cuts (first 0, last the band count). The chunk costs shrink
// geometrically (halving), since only the last chunk's copies are not hidden
// behind a later chunk's attention.
std::vector<int> push_chunks(const Split& s, int rank)
{
    const auto& rb = s.rank_bands[rank];
    double total = 0;
    for (int b : rb)
        total += s.bands[b].cost;
    const int chunks = std::max(1, std::min<int>(kPushChunks, (int)rb.size()));
    // shares 2^(chunks-1) : ... : 2 : 1 of the cost, cumulative targets
    std::vector<double> target;
    double sum = 0, unit = total / ((1 << chunks) - 1);
    for (int c = 0; c < chunks - 1; c++)
    {
        sum += unit * (1 << (chunks - 1 - c));
        target.push_back(sum);
    }
    std::vector<int> cuts{0};
    double acc = 0;
    for (size_t i = 0; i < rb.size(); i++)
    {
        acc += s.bands[rb[i]].cost;
        const size_t c = cuts.size() - 1;
        if (c < target.size() && i + 1 < rb.size() && acc >= target[c])
            cuts.push_back((int)i + 1);
    }
    cuts.push_back((int)rb.size());
    return cuts;
}

// Copies token runs of video rows from `local` into every peer at the same
// offsets, once the work enqueued so far on `st` is done: each peer's copies on
// its own stream. A run is one contiguous byte range (its tokens' rows and the
// padding between them), so each goes as a single peer copy.
int push_runs(awa_comm* c, const std::vector<std::pair<int64_t, int64_t>>& runs, unsigned char* local,
              const std::vector<unsigned char*>& peers, int64_t token_bytes, int64_t row_bytes, size_t chunk,
              cudaStream_t st)
{
    cudaError_t e = cudaEventRecord(c->chunk_ready[chunk], st);
    for (size_t q = 0; q < peers.size() && e == cudaSuccess; q++)
    {
        e = cudaStreamWaitEvent(c->push_stream[q], c->chunk_ready[chunk], 0);
        for (const auto& run : runs)
        {
            const int64_t off = run.first * token_bytes, bytes = (run.second - 1) * token_bytes + row_bytes;
            if (e == cudaSuccess)
                e = cudaMemcpyAsync(peers[q] + off, local + off, (size_t)bytes, cudaMemcpyDeviceToDevice,
                                    c->push_stream[q]);
        }
    }
    return cuda_status(e, "peer copy of video rows");
}

// `st` waits for every peer copy issued so far.
int join_pushes(awa_comm* c, cudaStream_t st)
{
    cudaError_t e = cudaSuccess;
    for (size_t q = 0; q < c->push_stream.size() && e == cudaSuccess; q++)
    {
        e = cudaEventRecord(c->push_done[q], c->push_stream[q]);
        if (e == cudaSuccess)
            e = cudaStreamWaitEvent(st, c->push_done[q], 0);
    }
    return cuda_status(e, "peer copy join");
}

// Pushes token runs into every peer with the SM copy kernel on `st` (after the
// work enqueued there), in launches of at most kMaxPushRuns runs.
int push_runs_kernel(const std::vector<std::pair<int64_t, int64_t>>& runs, unsigned char* local,
                     const std::vector<unsigned char*>& peers, int64_t token_bytes, int64_t row_bytes, cudaStream_t st)
{
    awa::PushPeers pp{};
    pp.count = (int)peers.size();
    for (size_t q = 0; q < peers.size(); q++)
        pp.ptr[q] = reinterpret_cast<uint4*>(peers[q]);
    size_t i = 0;
    while (i < runs.size())
    {
        awa::PushRuns pr{};
        for (; i < runs.size() && pr.n < awa::kMaxPushRuns; i++, pr.n++)
        {
            pr.first[pr.n] = runs[i].first * token_bytes / 16;
            pr.count[pr.n] = ((runs[i].second - 1) * token_bytes + row_bytes) / 16;
        }
        const int e = awa::launch_push_runs(local, pp, pr, st);
        if (e)
            return cuda_status(static_cast<cudaError_t>(e), "peer push kernel");
    }
    return AWA_OK;
}

}  // namespace

extern "C" {

int awa_comm_set_push(awa_comm* comm, int mode)
{
    if (!comm || (mode != AWA_PUSH_AUTO && mode != AWA_PUSH_COPY_ENGINES && mode != AWA_PUSH_KERNEL))
        return fail(AWA_ERR_INVALID, "awa_comm_set_push: unknown mode %d", mode);
    comm->push_mode = mode;
    return AWA_OK;
}

int awa_comm_alloc_shared(awa_comm* comm, size_t bytes, void** out)
{
    if (!comm || !out || bytes == 0)
        return fail(AWA_ERR_INVALID, "awa_comm_alloc_shared: invalid arguments");
    *out = nullptr;
    const Nccl* n = nccl();
    if (!n)
        return fail(AWA_ERR_CUDA, "awa_comm_alloc_shared: libnccl.so.2 could not be loaded");
    const int R = comm->nranks;
    // what each rank publishes: its buffer's IPC handle and size (every rank's
    // buffer must have the same size, since peers write at the writer's offsets)
    struct Record
    {
        cudaIpcMemHandle_t handle;
        uint64_t bytes;
    };
    SharedBuffer b;
    b.bytes = bytes;
    b.peer.assign(R, nullptr);
    unsigned char* records = nullptr;
    cudaStream_t st = nullptr;
    Record mine{};
    mine.bytes = bytes;
    cudaError_t e = cudaMalloc(&b.local, bytes);
    if (e == cudaSuccess)
        e = cudaMemset(b.local, 0, bytes);
    if (e == cudaSuccess)
        e = cudaIpcGetMemHandle(&mine.handle, b.local);
    if (e == cudaSuccess)
        e = cudaMalloc(&records, (size_t)R * sizeof(Record));
    if (e == cudaSuccess)
        e = cudaMemcpy(records + comm->rank * sizeof(Record), &mine, sizeof(Record), cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    int rc = cuda_status(e, "awa_comm_alloc_shared");
    if (rc == AWA_OK)
        rc = nccl_status(n, n->all_gather(records + comm->rank * sizeof(Record), records, sizeof(Record), ncclUint8,
                                          comm->comm, st),
                         "ncclAllGather (IPC handles)");
    std::vector<Record> all(R);
    if (rc == AWA_OK)
        rc = cuda_status(cudaStreamSynchronize(st), "awa_comm_alloc_shared");
    if (rc == AWA_OK)
        rc = cuda_status(cudaMemcpy(all.data(), records, (size_t)R * sizeof(Record), cudaMemcpyDeviceToHost),
                         "awa_comm_alloc_shared");
    for (int q = 0; q < R && rc == AWA_OK; q++)
        if (all[q].bytes != bytes)
            rc = fail(AWA_ERR_INVALID, "awa_comm_alloc_shared: rank %d asked for %llu bytes, rank %d for %zu", q,
                      (unsigned long long)all[q].bytes, comm->rank, bytes);
    for (int q = 0; q < R && rc == AWA_OK; q++)
    {
        if (q == comm->rank)
        {
            b.peer[q] = b.local;
            continue;
        }
        rc = cuda_status(cudaIpcOpenMemHandle(&b.peer[q], all[q].handle, cudaIpcMemLazyEnablePeerAccess),
                         "cudaIpcOpenMemHandle");
    }
    if (st)
        cudaStreamDestroy(st);
    if (records)
        cudaFree(records);
    if (rc != AWA_OK)
    {
        release_shared(b, comm->rank);
        return rc;
    }
    comm->shared.push_back(b);
    *out = b.local;
    return AWA_OK;
}

int awa_comm_free_shared(awa_comm* comm, void* ptr)
{
    if (!comm || !ptr)
        return fail(AWA_ERR_INVALID, "awa_comm_free_shared: invalid arguments");
    const Nccl* n = nccl();
    if (!n)
        return fail(AWA_ERR_CUDA, "awa_comm_free_shared: libnccl.so.2 could not be loaded");
    for (size_t i = 0; i < comm->shared.size(); i++)
        if (comm->shared[i].local == ptr)
        {
            // no rank may still be writing into another's buffer: finish this
            // rank's work, then wait for every rank
            int rc = cuda_status(cudaDeviceSynchronize(), "awa_comm_free_shared");
            if (rc == AWA_OK)
                rc = barrier(n, comm, nullptr);
            if (rc == AWA_OK)
                rc = cuda_status(cudaDeviceSynchronize(), "awa_comm_free_shared");
            release_shared(comm->shared[i], comm->rank);
            comm->shared.erase(comm->shared.begin() + i);
            return rc;
        }
    return fail(AWA_ERR_INVALID, "awa_comm_free_shared: not a buffer of this communicator");
}

int awa_comm_unique_id(unsigned char* id, size_t capacity)
{
    const Nccl* n = nccl();
    if (!n)
        return fail(AWA_ERR_CUDA, "awa_comm_unique_id: libnccl.so.2 could not be loaded");
    if (!id || capacity < sizeof(ncclUniqueId))
        return fail(AWA_ERR_INVALID, "awa_comm_unique_id: needs %zu bytes", sizeof(ncclUniqueId));
    ncclUniqueId uid;
    int rc = nccl_status(n, n->get_unique_id(&uid), "ncclGetUniqueId");
    if (rc == AWA_OK)
        std::memcpy(id, &uid, sizeof(uid));
    return rc;
}

int awa_comm_create(const unsigned char* id, size_t id_bytes, int nranks, int rank, awa_comm** out)
{
    if (!out)
        return fail(AWA_ERR_INVALID, "awa_comm_create: NULL output");
    *out = nullptr;
    const Nccl* n = nccl();
    if (!n)
        return fail(AWA_ERR_CUDA, "awa_comm_create: libnccl.so.2 could not be loaded");
    if (!id || id_bytes < sizeof(ncclUniqueId) || nranks <= 0 || rank < 0 || rank >= nranks)
        return fail(AWA_ERR_INVALID, "awa_comm_create: invalid id, rank %d or nranks %d", rank, nranks);
    awa_comm* c = new awa_comm();
    if (cudaGetDevice(&c->device) != cudaSuccess)
    {
        delete c;
        return fail(AWA_ERR_CUDA, "awa_comm_create: no current device");
    }
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    const int rc = nccl_status(n, n->comm_init_rank(&c->comm, nranks, uid, rank), "ncclCommInitRank");
    if (rc != AWA_OK)
    {
        delete c;
        return rc;
    }
    c->rank = rank;
    c->nranks = nranks;
    c->owned = true;
    if (cudaMalloc(&c->barrier_word, sizeof(int)) != cudaSuccess ||
        cudaMemset(c->barrier_word, 0, sizeof(int)) != cudaSuccess)
    {
        n->comm_destroy(c->comm);
        delete c;
        return fail(AWA_ERR_ALLOC, "awa_comm_create: device allocation failed");
    }
    *out = c;
    return AWA_OK;
}

int awa_comm_wrap(void* nccl_comm, awa_comm** out)
{
    if (!out || !nccl_comm)
        return fail(AWA_ERR_INVALID, "awa_comm_wrap: NULL communicator");
    *out = nullptr;
    const Nccl* n = nccl();
    if (!n)
        return fail(AWA_ERR_CUDA, "awa_comm_wrap: libnccl.so.2 could not be loaded");
    awa_comm* c = new awa_comm();
    c->comm = static_cast<ncclComm_t>(nccl_comm);
    int rc = nccl_status(n, n->comm_count(c->comm, &c->nranks), "ncclCommCount");
    if (rc == AWA_OK)
        rc = nccl_status(n, n->comm_user_rank(c->comm, &c->rank), "ncclCommUserRank");
    if (rc == AWA_OK && cudaGetDevice(&c->device) != cudaSuccess)
        rc = fail(AWA_ERR_CUDA, "awa_comm_wrap: no current device");
    if (rc == AWA_OK && (cudaMalloc(&c->barrier_word, sizeof(int)) != cudaSuccess ||
                         cudaMemset(c->barrier_word, 0, sizeof(int)) != cudaSuccess))
        rc = fail(AWA_ERR_ALLOC, "awa_comm_wrap: device allocation failed");
    if (rc != AWA_OK)
    {
        delete c;
        return rc;
    }
    *out = c;
    return AWA_OK;
}

void awa_comm_destroy(awa_comm* comm)
{
    if (!comm)
        return;
    for (SharedBuffer& b : comm->shared)
        release_shared(b, comm->rank);
    if (comm->barrier_word)
        cudaFree(comm->barrier_word);
    for (cudaEvent_t e : comm->chunk_ready)
        if (e)
            cudaEventDestroy(e);
    for (cudaEvent_t e : comm->push_done)
        if (e)
            cudaEventDestroy(e);
    for (cudaStream_t s : comm->push_stream)
        if (s)
            cudaStreamDestroy(s);
    const Nccl* n = nccl();
    if (comm->owned && comm->comm && n)
        n->comm_destroy(comm->comm);
    delete comm;
}

int awa_comm_info(const awa_comm* comm, int* rank, int* nranks)
{
    if (!comm)
        return fail(AWA_ERR_INVALID, "awa_comm_info: NULL communicator");
    if (rank)
        *rank = comm->rank;
    if (nranks)
        *nranks = comm->nranks;
    return AWA_OK;
}

int awa_shard_split(const awa_plan* plan, int nranks, int heads, int* by_heads, int* bounds)
{
    awa_plan_info info;
    if (!plan || nranks <= 0 || heads <= 0 || awa_plan_get_info(plan, &info) != AWA_OK)
        return fail(AWA_ERR_INVALID, "awa_shard_split: invalid arguments");
    const Split s = make_split(plan, info, nranks, heads);
    if (by_heads)
        *by_heads = s.by_heads ? 1 : 0;
    if (bounds)
        std::copy(s.bounds.begin(), s.bounds.end(), bounds);
    return AWA_OK;
}

int awa_shard_windows(const awa_plan* plan, int nranks, int heads, int rank, int* windows, int capacity)
{
    awa_plan_info info;
    if (!plan || nranks <= 0 || heads <= 0 || rank < 0 || rank >= nranks || capacity < 0 ||
        (capacity > 0 && !windows) || awa_plan_get_info(plan, &info) != AWA_OK)
        return fail(AWA_ERR_INVALID, "awa_shard_windows: invalid arguments");
    const Split s = make_split(plan, info, nranks, heads);
    if (s.by_heads)
    {
        for (int w = 0; w < std::min(capacity, info.window_count); w++)
            windows[w] = w;
        return info.window_count;
    }
    const auto& mine = s.windows[rank];
    std::copy(mine.begin(), mine.begin() + std::min<size_t>(capacity, mine.size()), windows);
    return (int)mine.size();
}

int awa_shard_runs(const awa_plan* plan, int nranks, int heads, int rank, int64_t* runs, int capacity)
{
    awa_plan_info info;
    if (!plan || nranks <= 0 || heads <= 0 || rank < 0 || rank >= nranks || capacity < 0 ||
        (capacity > 0 && !runs) || awa_plan_get_info(plan, &info) != AWA_OK)
        return fail(AWA_ERR_INVALID, "awa_shard_runs: invalid arguments");
    const Split s = make_split(plan, info, nranks, heads);
    std::vector<std::pair<int64_t, int64_t>> mine;
    if (s.by_heads)
        mine.emplace_back(0, info.source_tokens);  // every token (a head slice of each row)
    else
        mine = band_runs(s, info, s.rank_bands[rank].data(), (int)s.rank_bands[rank].size());
    for (size_t i = 0; i < mine.size() && (int)i < capacity; i++)
    {
        runs[2 * i] = mine[i].first;
        runs[2 * i + 1] = mine[i].second;
    }
    return (int)mine.size();
}

size_t awa_forward_sharded_workspace_bytes(const awa_plan* plan, int nranks, int heads, int head_dim, int out_dtype)
{
    awa_plan_info info;
    if (!plan || nranks <= 0 || heads <= 0 || head_dim <= 0 || awa_plan_get_info(plan, &info) != AWA_OK)
        return 0;
    const Split s = make_split(plan, info, nranks, heads);
    return make_layout(plan, info, s, nranks, heads, head_dim, out_dtype).total;
}

int awa_forward_sharded(const awa_plan* plan, awa_comm* comm, int precision, int heads, int head_dim, int in_dtype,
                        const void* video_qkv, int64_t video_token_stride, int64_t video_qkv_stride,
                        const void* text_qkv, int64_t text_token_stride, int64_t text_qkv_stride, int out_dtype,
                        void* video_out, int64_t video_token_stride_out, void* text_out,
                        int64_t text_token_stride_out, void* workspace, size_t workspace_bytes, awa_stream_t stream)
{
    awa_plan_info info;
    if (!plan || !comm || awa_plan_get_info(plan, &info) != AWA_OK)
        return fail(AWA_ERR_INVALID, "awa_forward_sharded: NULL plan or communicator");
    if (heads <= 0 || head_dim <= 0 || !video_qkv || !text_qkv || !video_out || !text_out || !workspace ||
        (out_dtype != AWA_F32 && out_dtype != AWA_BF16) || video_token_stride_out < (int64_t)heads * head_dim)
        return fail(AWA_ERR_INVALID, "awa_forward_sharded: invalid arguments");
    int device = -1;
    if (cudaGetDevice(&device) != cudaSuccess || device != comm->device || device != info.device)
        return fail(AWA_ERR_INVALID, "awa_forward_sharded: plan, communicator and current device differ");
    const Nccl* n = nccl();
    if (!n)
        return fail(AWA_ERR_CUDA, "awa_forward_sharded: libnccl.so.2 could not be loaded");
    const int R = comm->nranks, r = comm->rank;
    const Split s = make_split(plan, info, R, heads);
    const Layout l = make_layout(plan, info, s, R, heads, head_dim, out_dtype);
    if (workspace_bytes < l.total)
        return fail(AWA_ERR_INVALID, "awa_forward_sharded: workspace of %zu bytes needed, %zu given", l.total,
                    workspace_bytes);
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t osz = dsize(out_dtype), isz = dsize(in_dtype);
    const ncclDataType_t otype = out_dtype == AWA_BF16 ? ncclBfloat16 : ncclFloat32;
    const int64_t row = (int64_t)heads * head_dim;
    int rc = AWA_OK;

    // Direct mode: video_out lies in a buffer shared over the ranks. This
    // rank's video rows then go straight into every other rank's copy of
    // video_out over NVLink, with no all-gather, staging or scatter: with one
    // peer the copy engines push them chunk by chunk as the attention kernel
    // finishes them (peer copies on side streams, overlapping the next chunk's
    // attention); with more peers (or when asked) the SM push kernel pushes
    // them after the attention. An entry barrier keeps any rank from writing
    // before every rank is done with the previous contents; the text
    // collective at the end, enqueued after the pushes, orders them before
    // every rank's later reads.
    const size_t video_span = (size_t)(info.source_tokens - 1) * video_token_stride_out * osz + (size_t)row * osz;
    const SharedBuffer* shared = find_shared(comm, video_out, video_span);
    const bool direct = shared != nullptr && R > 1;
    std::vector<unsigned char*> peers;  // the other ranks' video_out
    if (direct)
    {
        const size_t off = static_cast<unsigned char*>(video_out) - static_cast<unsigned char*>(shared->local);
        for (int q = 0; q < R; q++)
            if (q != r)
                peers.push_back(static_cast<unsigned char*>(shared->peer[q]) + off);
        if ((rc = push_streams(comm)) != AWA_OK || (rc = barrier(n, comm, st)) != AWA_OK)
            return rc;
    }

    if (s.by_heads)
    {
        // This rank's heads [h0, h1) over every window: offset pointers, same strides.
        const int h0 = s.bounds[r], hn = s.bounds[r + 1] - s.bounds[r];
        int most = 0;
        for (int q = 0; q < R; q++)
            most = std::max(most, s.bounds[q + 1] - s.bounds[q]);
        const size_t hoff_in = (size_t)h0 * head_dim * isz, hoff_out = (size_t)h0 * head_dim * osz;
        if (hn > 0)
            rc = awa_forward(plan, precision, hn, head_dim, in_dtype,
                             static_cast<const unsigned char*>(video_qkv) + hoff_in, video_token_stride,
                             video_qkv_stride, static_cast<const unsigned char*>(text_qkv) + hoff_in,
                             text_token_stride, text_qkv_stride, out_dtype,
                             static_cast<unsigned char*>(video_out) + hoff_out, video_token_stride_out,
                             static_cast<unsigned char*>(text_out) + hoff_out, text_token_stride_out,
                             ws + l.forward, l.gather - l.forward, stream);
        if (rc)
            return rc;
        const size_t vslot = (size_t)info.source_tokens * most * head_dim, tslot = (size_t)info.text_tokens * most * head_dim;
        unsigned char* vg = ws + l.gather;
        unsigned char* tg = ws + l.text_gather;
        const size_t width = (size_t)hn * head_dim * osz, spitch = (size_t)most * head_dim * osz;
        const size_t vpitch = (size_t)video_token_stride_out * osz;
        if (hn > 0 && direct)
            // the head slice of every token row, into every peer's output
            for (unsigned char* peer : peers)
                if (rc == AWA_OK)
                    rc = cuda_status(cudaMemcpy2DAsync(peer + hoff_out, vpitch,
                                                       static_cast<unsigned char*>(video_out) + hoff_out, vpitch,
                                                       width, info.source_tokens, cudaMemcpyDeviceToDevice, st),
                                     "head slice push (video)");
        if (hn > 0 && !direct && rc == AWA_OK)
            rc = cuda_status(cudaMemcpy2DAsync(vg + r * vslot * osz, spitch,
                                               static_cast<unsigned char*>(video_out) + hoff_out, vpitch, width,
                                               info.source_tokens, cudaMemcpyDeviceToDevice, st),
                             "head slice pack (video)");
        if (hn > 0 && rc == AWA_OK)
            rc = cuda_status(cudaMemcpy2DAsync(tg + r * tslot * osz, spitch,
                                               static_cast<unsigned char*>(text_out) + hoff_out,
                                               text_token_stride_out * osz, width, info.text_tokens,
                                               cudaMemcpyDeviceToDevice, st),
                             "head slice pack (text)");
        if (rc)
            return rc;
        rc = nccl_status(n, n->group_start(), "ncclGroupStart");
        if (rc == AWA_OK && !direct)
            rc = nccl_status(n, n->all_gather(vg + r * vslot * osz, vg, vslot, otype, comm->comm, st),
                             "ncclAllGather (video)");
        if (rc == AWA_OK)
            rc = nccl_status(n, n->all_gather(tg + r * tslot * osz, tg, tslot, otype, comm->comm, st),
                             "ncclAllGather (text)");
        const int end_rc = nccl_status(n, n->group_end(), "ncclGroupEnd");
        rc = rc ? rc : end_rc;
        for (int q = 0; q < R && rc == AWA_OK; q++)
        {
            const int qn = s.bounds[q + 1] - s.bounds[q];
            if (q == r || qn == 0)
                continue;
            const size_t qoff = (size_t)s.bounds[q] * head_dim * osz, qwidth = (size_t)qn * head_dim * osz;
            if (!direct)
                rc = cuda_status(cudaMemcpy2DAsync(static_cast<unsigned char*>(video_out) + qoff, vpitch,
                                                   vg + q * vslot * osz, spitch, qwidth, info.source_tokens,
                                                   cudaMemcpyDeviceToDevice, st),
                                 "head slice unpack (video)");
            if (rc == AWA_OK)
                rc = cuda_status(cudaMemcpy2DAsync(static_cast<unsigned char*>(text_out) + qoff,
                                                   text_token_stride_out * osz, tg + q * tslot * osz, spitch, qwidth,
                                                   info.text_tokens, cudaMemcpyDeviceToDevice, st),
                                 "head slice unpack (text)");
        }
        return rc;
    }

    // Window split: this rank's bands (whole grid lines of every frame they span).
    const std::vector<int>& mine = s.windows[r];
    const int64_t tbytes = video_token_stride_out * (int64_t)osz, rbytes = row * (int64_t)osz;
    float* text_sum = reinterpret_cast<float*>(ws + l.text_sum);
    unsigned char* partials = ws + l.forward;
    const size_t partial_bytes = l.gather - l.forward;
    const size_t window_partial = (size_t)info.text_tokens * row;  // elements per window
    int partial_dtype = AWA_F32;
    const int64_t rank_units_ok = tbytes % 16 == 0 && rbytes % 16 == 0 &&
                                  reinterpret_cast<uintptr_t>(video_out) % 16 == 0;
    const bool push_kernel = direct && rank_units_ok &&
                             (comm->push_mode == AWA_PUSH_KERNEL ||
                              (comm->push_mode == AWA_PUSH_AUTO && (int)peers.size() >= 3));
    if (direct && push_kernel)
    {
        // one attention launch over the rank's windows, then the SM copy kernel
        // pushes its rows into every peer (NVLink stores from all SMs)
        const auto& rb = s.rank_bands[r];
        rc = awa::attention_set(plan, precision, heads, head_dim, mine.data(), (int)mine.size(), in_dtype, video_qkv,
                                video_token_stride, video_qkv_stride, text_qkv, text_token_stride, text_qkv_stride,
                                out_dtype, video_out, video_token_stride_out, partials, partial_bytes, &partial_dtype,
                                st);
        if (rc == AWA_OK)
            rc = push_runs_kernel(band_runs(s, info, rb.data(), (int)rb.size()), static_cast<unsigned char*>(video_out),
                                  peers, tbytes, rbytes, st);
        if (rc == AWA_OK)
            rc = awa::text_partial_sum(plan, heads, head_dim, partial_dtype, partials, 0, (int)mine.size(), text_sum,
                                       st);
        if (rc == AWA_OK)
            rc = nccl_status(n, n->all_reduce(text_sum, text_sum, (size_t)info.text_tokens * row, ncclFloat32, ncclSum,
                                              comm->comm, st),
                             "ncclAllReduce (text partial sums)");
        if (rc)
            return rc;
        return awa_text_finalize(plan, heads, head_dim, text_sum, out_dtype, text_out, text_token_stride_out, stream);
    }
    if (direct)
    {
        // chunk by chunk: attention of the chunk's windows, then its rows to the
        // peers on the copy engines while the next chunk computes
        const std::vector<int> cuts = push_chunks(s, r);
        const auto& rb = s.rank_bands[r];
        const size_t psz = awa_attention_kernel_kind(plan, precision, in_dtype, heads, head_dim) == 1 ? 2 : 4;
        size_t done = 0;  // windows (partial slots) of the chunks so far
        for (size_t c = 0; c + 1 < cuts.size() && rc == AWA_OK; c++)
        {
            const std::vector<int> set = band_windows(s, rb.data() + cuts[c], cuts[c + 1] - cuts[c]);
            const size_t off = done * window_partial * psz;
            rc = awa::attention_set(plan, precision, heads, head_dim, set.data(), (int)set.size(), in_dtype,
                                    video_qkv, video_token_stride, video_qkv_stride, text_qkv, text_token_stride,
                                    text_qkv_stride, out_dtype, video_out, video_token_stride_out, partials + off,
                                    partial_bytes - off, &partial_dtype, st);
            done += set.size();
            if (rc == AWA_OK)
                rc = push_runs(comm, band_runs(s, info, rb.data() + cuts[c], cuts[c + 1] - cuts[c]),
                               static_cast<unsigned char*>(video_out), peers, tbytes, rbytes, c, st);
        }
        // the chunks' partial slots run in band order; the sum over all of them
        // covers this rank's windows once each
        if (rc == AWA_OK)
            rc = awa::text_partial_sum(plan, heads, head_dim, partial_dtype, partials, 0, (int)done, text_sum, st);
        if (rc == AWA_OK)
            rc = join_pushes(comm, st);
        if (rc == AWA_OK)
            rc = nccl_status(n, n->all_reduce(text_sum, text_sum, (size_t)info.text_tokens * row, ncclFloat32, ncclSum,
                                              comm->comm, st),
                             "ncclAllReduce (text partial sums)");
        if (rc)
            return rc;
        return awa_text_finalize(plan, heads, head_dim, text_sum, out_dtype, text_out, text_token_stride_out, stream);
    }

    // All-gather mode: attention of this rank's windows, its runs packed into its
    // slot of the gather buffer, NCCL all-gather of the slots and all-reduce of
    // the text partial sums, the other ranks' runs copied back into place.
    rc = awa::attention_set(plan, precision, heads, head_dim, mine.data(), (int)mine.size(), in_dtype, video_qkv,
                            video_token_stride, video_qkv_stride, text_qkv, text_token_stride, text_qkv_stride,
                            out_dtype, video_out, video_token_stride_out, partials, partial_bytes, &partial_dtype, st);
    if (rc == AWA_OK)
        rc = awa::text_partial_sum(plan, heads, head_dim, partial_dtype, partials, 0, (int)mine.size(), text_sum, st);
    if (rc)
        return rc;
    unsigned char* gather = ws + l.gather;
    const size_t slot_bytes = (size_t)std::max<int64_t>(s.slot_rows, 1) * rbytes;  // dense rows
    auto copy_runs = [&](int q, bool to_slot) {
        const auto runs = band_runs(s, info, s.rank_bands[q].data(), (int)s.rank_bands[q].size());
        unsigned char* slot = gather + q * slot_bytes;
        int64_t at = 0;
        int result = AWA_OK;
        for (const auto& run : runs)
        {
            unsigned char* v = static_cast<unsigned char*>(video_out) + run.first * tbytes;
            if (result == AWA_OK)
                result = cuda_status(to_slot ? cudaMemcpy2DAsync(slot + at, rbytes, v, tbytes, rbytes, run.second,
                                                                 cudaMemcpyDeviceToDevice, st)
                                             : cudaMemcpy2DAsync(v, tbytes, slot + at, rbytes, rbytes, run.second,
                                                                 cudaMemcpyDeviceToDevice, st),
                                     "video run copy");
            at += run.second * rbytes;
        }
        return result;
    };
    rc = copy_runs(r, true);
    if (rc)
        return rc;
    rc = nccl_status(n, n->group_start(), "ncclGroupStart");
    if (rc == AWA_OK)
        rc = nccl_status(n, n->all_reduce(text_sum, text_sum, (size_t)info.text_tokens * row, ncclFloat32, ncclSum,
                                          comm->comm, st),
                         "ncclAllReduce (text partial sums)");
    if (rc == AWA_OK)
        rc = nccl_status(n, n->all_gather(gather + r * slot_bytes, gather, slot_bytes / osz, otype, comm->comm, st),
                         "ncclAllGather (video rows)");
    const int end_rc = nccl_status(n, n->group_end(), "ncclGroupEnd");
    rc = rc ? rc : end_rc;
    if (rc)
        return rc;
    rc = awa_text_finalize(plan, heads, head_dim, text_sum, out_dtype, text_out, text_token_stride_out, stream);
    for (int q = 0; q < R && rc == AWA_OK; q++)
        if (q != r)
            rc = copy_runs(q, false);
    return rc;
}

}  // extern "C"
