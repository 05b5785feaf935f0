// awa_shard.cpp -- one AWA layer split over the GPUs of a node
// (include/awa_b200.h: awa_comm_*, awa_forward_sharded).
//
// Windows are independent (SeedVR2WindowAttention::forward runs each window on
// its own, awa_layers.cpp:1062-1120); the only coupling between them is the
// text mean text[i] = sum_w attended_text(w)[i] / W (awa_layers.cpp:684-685).
// So each rank computes a share of the layer and two collectives finish it:
//
//   window split (enough windows): rank r runs the fused forward on a
//     contiguous range of windows of near-equal attention cost, packs its
//     video rows into its slot of a gather buffer, NCCL all-gathers the slots
//     (in place), all-reduces the fp32 text partial sums and scatters the other
//     ranks' rows into its own video output;
//   head split (fewer than 4 windows per rank): rank r runs the whole layer for
//     a range of heads -- the QKV and output pointers offset by the first head,
//     the row strides unchanged -- and the all-gather moves head slices of the
//     video and text outputs.
//
// Every rank ends with the full video and text outputs, as the ncnn boundary
// requires. NCCL moves the data into local memory: no kernel reads a peer's
// memory and nothing uses TMA multicast. libnccl.so.2 is opened at run time,
// so the library loads on machines without NCCL; inside a PyTorch process the
// dynamic loader hands back the NCCL that torch already loaded.
#include "awa_b200.h"
#include "awa_internal.h"

#include <dlfcn.h>

#include <nccl.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
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
    cudaStream_t push_stream = nullptr;  // direct mode: peer copies of video rows
    cudaEvent_t push_events[8] = {};     // per chunk, and the join
};

namespace
{

// How one layer is split over the ranks of a communicator.
struct Split
{
    bool by_heads = false;
    std::vector<int> bounds;  // window bounds (nranks + 1) or head bounds (nranks + 1)
    int64_t slot_rows = 0;    // window split: rows of one rank's slot of the gather buffer
};

Split make_split(const awa_plan* plan, const awa_plan_info& info, int nranks, int heads)
{
    Split s;
    s.bounds.assign(nranks + 1, 0);
    s.by_heads = nranks > 1 && info.window_count < 4 * nranks && heads >= nranks;
    if (s.by_heads)
    {
        for (int r = 0; r <= nranks; r++)
            s.bounds[r] = (int)((int64_t)heads * r / nranks);
        return s;
    }
    awa_partition_windows(plan, nranks, s.bounds.data());
    for (int r = 0; r < nranks; r++)
        s.slot_rows = std::max<int64_t>(s.slot_rows, awa_window_range_video_rows(plan, s.bounds[r], s.bounds[r + 1]));
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
        int most = 0;
        for (int r = 0; r < nranks; r++)
            most = std::max(most, s.bounds[r + 1] - s.bounds[r]);
        off += align256((size_t)std::max(most, 1) * info.text_tokens * row * sizeof(float));
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
constexpr int kPushChunks = 4;  // attention launches per rank, each followed by its rows' peer copies

// The side stream and events of the peer copies (made once per communicator).
int push_streams(awa_comm* c)
{
    if (c->push_stream)
        return AWA_OK;
    cudaError_t e = cudaStreamCreateWithFlags(&c->push_stream, cudaStreamNonBlocking);
    for (int i = 0; i < kPushChunks + 1 && e == cudaSuccess; i++)
        e = cudaEventCreateWithFlags(&c->push_events[i], cudaEventDisableTiming);
    return cuda_status(e, "peer copy stream");
}

// Chunk boundaries of windows [w0, w1): up to kPushChunks runs of near-equal
// attention cost (sum of L^2, L = video rows; the text rows add the same to
// every window of one shape).
std::vector<int> push_chunks(const std::vector<awa_window>& win, int w0, int w1)
{
    std::vector<double> cost;
    double total = 0;
    for (int w = w0; w < w1; w++)
    {
        const double L = (double)(win[w].t1 - win[w].t0) * (win[w].h1 - win[w].h0) * (win[w].w1 - win[w].w0);
        cost.push_back(L * L);
        total += L * L;
    }
    const int chunks = std::max(1, std::min(kPushChunks, (w1 - w0) / 8));
    std::vector<int> cuts{w0};
    double acc = 0;
    int w = w0;
    for (int c = 1; c < chunks; c++)
    {
        while (w < w1 && acc + 0.5 * cost[w - w0] < total * c / chunks)
            acc += cost[w++ - w0];
        if (w > cuts.back())
            cuts.push_back(w);
    }
    if (w1 > cuts.back())
        cuts.push_back(w1);
    return cuts;
}

// Copies the video rows of windows [wb, we) from `local` into every peer, on
// the side stream once the attention that wrote them (enqueued on `st`) is
// done. Windows in plan order run t fastest, then h, then w: runs of windows
// are merged into boxes (t0..t1, h0..h1, w0..w1) first along t, then h, then w,
// and each box goes as one pitched copy per frame per peer.
int push_rows(awa_comm* c, const std::vector<awa_window>& win, int wb, int we, unsigned char* local,
              const std::vector<unsigned char*>& peers, int64_t line_bytes, int64_t frame_bytes, int64_t token_bytes,
              int64_t row_bytes, size_t chunk, cudaStream_t st)
{
    std::vector<awa_window> boxes;
    for (int w = wb; w < we; w++)
    {
        const awa_window& x = win[w];
        if (!boxes.empty())
        {
            awa_window& b = boxes.back();
            if (b.h0 == x.h0 && b.h1 == x.h1 && b.w0 == x.w0 && b.w1 == x.w1 && b.t1 == x.t0)
            {
                b.t1 = x.t1;
                continue;
            }
            if (b.t0 == x.t0 && b.t1 == x.t1 && b.w0 == x.w0 && b.w1 == x.w1 && b.h1 == x.h0)
            {
                b.h1 = x.h1;
                continue;
            }
        }
        boxes.push_back(x);
    }
    // boxes that follow each other along w
    std::vector<awa_window> merged;
    for (const awa_window& x : boxes)
    {
        if (!merged.empty())
        {
            awa_window& b = merged.back();
            if (b.t0 == x.t0 && b.t1 == x.t1 && b.h0 == x.h0 && b.h1 == x.h1 && b.w1 == x.w0)
            {
                b.w1 = x.w1;
                continue;
            }
        }
        merged.push_back(x);
    }
    cudaError_t e = cudaEventRecord(c->push_events[chunk], st);
    if (e == cudaSuccess)
        e = cudaStreamWaitEvent(c->push_stream, c->push_events[chunk], 0);
    for (const awa_window& b : merged)
    {
        const int64_t width = (int64_t)(b.w1 - b.w0 - 1) * token_bytes + row_bytes;
        for (int t = b.t0; t < b.t1 && e == cudaSuccess; t++)
        {
            const int64_t off = t * frame_bytes + b.h0 * line_bytes + b.w0 * token_bytes;
            for (unsigned char* peer : peers)
                if (e == cudaSuccess)
                    e = cudaMemcpy2DAsync(peer + off, line_bytes, local + off, line_bytes, width, b.h1 - b.h0,
                                          cudaMemcpyDeviceToDevice, c->push_stream);
        }
    }
    return cuda_status(e, "peer copy of video rows");
}

// `st` waits for every peer copy issued so far.
int join_pushes(awa_comm* c, cudaStream_t st)
{
    cudaError_t e = cudaEventRecord(c->push_events[kPushChunks], c->push_stream);
    if (e == cudaSuccess)
        e = cudaStreamWaitEvent(st, c->push_events[kPushChunks], 0);
    return cuda_status(e, "peer copy join");
}

}  // namespace

extern "C" {

int awa_comm_alloc_shared(awa_comm* comm, size_t bytes, void** out)
{
    if (!comm || !out || bytes == 0)
        return fail(AWA_ERR_INVALID, "awa_comm_alloc_shared: invalid arguments");
    *out = nullptr;
    const Nccl* n = nccl();
    if (!n)
        return fail(AWA_ERR_CUDA, "awa_comm_alloc_shared: libnccl.so.2 could not be loaded");
    const int R = comm->nranks;
    SharedBuffer b;
    b.bytes = bytes;
    b.peer.assign(R, nullptr);
    unsigned char* handles = nullptr;
    cudaStream_t st = nullptr;
    cudaError_t e = cudaMalloc(&b.local, bytes);
    if (e == cudaSuccess)
        e = cudaMemset(b.local, 0, bytes);
    cudaIpcMemHandle_t mine;
    if (e == cudaSuccess)
        e = cudaIpcGetMemHandle(&mine, b.local);
    if (e == cudaSuccess)
        e = cudaMalloc(&handles, (size_t)R * sizeof(cudaIpcMemHandle_t));
    if (e == cudaSuccess)
        e = cudaMemcpy(handles + comm->rank * sizeof(mine), &mine, sizeof(mine), cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    int rc = cuda_status(e, "awa_comm_alloc_shared");
    // every rank's handle to every rank
    if (rc == AWA_OK)
        rc = nccl_status(n, n->all_gather(handles + comm->rank * sizeof(mine), handles, sizeof(mine), ncclUint8,
                                          comm->comm, st),
                         "ncclAllGather (IPC handles)");
    std::vector<cudaIpcMemHandle_t> all(R);
    if (rc == AWA_OK)
        rc = cuda_status(cudaStreamSynchronize(st), "awa_comm_alloc_shared");
    if (rc == AWA_OK)
        rc = cuda_status(cudaMemcpy(all.data(), handles, (size_t)R * sizeof(mine), cudaMemcpyDeviceToHost),
                         "awa_comm_alloc_shared");
    for (int q = 0; q < R && rc == AWA_OK; q++)
    {
        if (q == comm->rank)
        {
            b.peer[q] = b.local;
            continue;
        }
        rc = cuda_status(cudaIpcOpenMemHandle(&b.peer[q], all[q], cudaIpcMemLazyEnablePeerAccess),
                         "cudaIpcOpenMemHandle");
    }
    if (st)
        cudaStreamDestroy(st);
    if (handles)
        cudaFree(handles);
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
    for (cudaEvent_t e : comm->push_events)
        if (e)
            cudaEventDestroy(e);
    if (comm->push_stream)
        cudaStreamDestroy(comm->push_stream);
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

    // Direct mode: video_out lies in a buffer shared over the ranks. The copy
    // engines then push this rank's video rows into every other rank's copy of
    // video_out over NVLink (peer copies on a side stream), chunk by chunk as
    // the attention kernel finishes them, so the transfer overlaps the next
    // chunk's attention and needs no all-gather, staging or scatter. An entry
    // barrier keeps any rank from writing before every rank is done with the
    // previous contents; the text collective at the end, enqueued after the
    // copies, orders them before every rank's later reads.
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
    const int64_t line_bytes = (int64_t)info.source_w * video_token_stride_out * osz;  // one grid line of tokens

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

    // Window split: this rank's windows [w0, w1).
    const int w0 = s.bounds[r], w1 = s.bounds[r + 1];
    float* text_sum = reinterpret_cast<float*>(ws + l.text_sum);
    unsigned char* partials = ws + l.forward;
    const size_t partial_bytes = l.gather - l.forward;
    const size_t window_partial = (size_t)info.text_tokens * row;  // elements per window
    int partial_dtype = AWA_F32;
    if (direct)
    {
        std::vector<awa_window> windows(info.window_count);
        awa_plan_get_maps(plan, nullptr, nullptr, nullptr, nullptr, windows.data());
        const std::vector<int> cuts = push_chunks(windows, w0, w1);
        for (size_t c = 0; c + 1 < cuts.size() && rc == AWA_OK; c++)
        {
            const int cb = cuts[c], ce = cuts[c + 1];
            int pd = AWA_F32;
            const size_t psz_guess = awa_attention_kernel_kind(plan, precision, in_dtype, heads, head_dim) == 1 ? 2 : 4;
            const size_t off = (size_t)(cb - w0) * window_partial * psz_guess;
            rc = awa::attention_range(plan, precision, heads, head_dim, cb, ce, in_dtype, video_qkv,
                                      video_token_stride, video_qkv_stride, text_qkv, text_token_stride,
                                      text_qkv_stride, out_dtype, video_out, video_token_stride_out, partials + off,
                                      partial_bytes - off, &pd, st);
            partial_dtype = pd;
            if (rc == AWA_OK)
                rc = push_rows(comm, windows, cb, ce, static_cast<unsigned char*>(video_out), peers, line_bytes,
                               (int64_t)info.source_h * line_bytes, video_token_stride_out * osz, row * osz, c, st);
        }
        if (rc == AWA_OK)
            rc = awa::text_partial_sum(plan, heads, head_dim, partial_dtype, partials, w0, w1, text_sum, st);
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

    rc = awa_forward_windows(plan, precision, heads, head_dim, w0, w1, in_dtype, video_qkv, video_token_stride,
                             video_qkv_stride, text_qkv, text_token_stride, text_qkv_stride, out_dtype, video_out,
                             video_token_stride_out, text_sum, partials, partial_bytes, stream);
    if (rc)
        return rc;
    unsigned char* gather = ws + l.gather;
    const size_t slot = (size_t)s.slot_rows * row;  // elements
    rc = awa_gather_video_shard(plan, heads, head_dim, w0, w1, out_dtype, video_out, video_token_stride_out,
                                gather + r * slot * osz, stream);
    if (rc)
        return rc;
    rc = nccl_status(n, n->group_start(), "ncclGroupStart");
    if (rc == AWA_OK)
        rc = nccl_status(n, n->all_reduce(text_sum, text_sum, (size_t)info.text_tokens * row, ncclFloat32, ncclSum,
                                          comm->comm, st),
                         "ncclAllReduce (text partial sums)");
    if (rc == AWA_OK && slot > 0)
        rc = nccl_status(n, n->all_gather(gather + r * slot * osz, gather, slot, otype, comm->comm, st),
                         "ncclAllGather (video rows)");
    const int end_rc = nccl_status(n, n->group_end(), "ncclGroupEnd");
    rc = rc ? rc : end_rc;
    if (rc)
        return rc;
    rc = awa_text_finalize(plan, heads, head_dim, text_sum, out_dtype, text_out, text_token_stride_out, stream);
    for (int q = 0; q < R && rc == AWA_OK; q++)
        if (q != r)
            rc = awa_scatter_video_shard(plan, heads, head_dim, s.bounds[q], s.bounds[q + 1], out_dtype,
                                         gather + q * slot * osz, video_out, video_token_stride_out, stream);
    return rc;
}

}  // extern "C"
