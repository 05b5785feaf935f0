/*
 * awa_b200.h -- C ABI of the B200 (sm_100a) adaptive window attention (AWA)
 * layers of SeedVR2. Drop-in for the four ncnn custom layers of
 * HGinkgo/SeedVR2-ncnn src/awa (SeedVR2AWAPack -> SeedVR2MMRoPE ->
 * SeedVR2WindowAttention -> SeedVR2AWAUnpack); the ncnn-compatible C++ layer
 * classes in seedvr2-ncnn_b200/ncnn_compat/ call these entry points.
 *
 * Conventions (same as the ncnn layers they replace):
 *   - status codes: 0 ok, -1 invalid shape / params / state, -100 allocation
 *     failure (awa_layers.cpp:411, 424, 439, 509); this library adds -2 for a
 *     CUDA runtime error and -3 for a device-side check that failed. The text
 *     of the last error of the calling thread is in awa_last_error().
 *   - every tensor argument is a DEVICE pointer on the plan's device, except
 *     where a function says "host"; strides are in elements, not bytes.
 *   - all work is enqueued on the given stream; nothing synchronises.
 *   - inputs are const; outputs are written completely (no accumulation).
 *   - the QKV blob of a layer is addressed as
 *       base + token * token_stride + qkv * qkv_stride + head * head_dim + f
 *     which covers every encoding describe_qkv_layout accepts
 *     (awa_layers.cpp:116-175): (w=d,h=3H,c=N) -> token_stride=cstep,
 *     qkv_stride=H*d; (w=d,h=H,c=3N) -> token_stride=cstep, qkv_stride=N*cstep;
 *     (w=d,h=H,d=3,c=N) -> token_stride=cstep, qkv_stride=H*d.
 *   - packed / attended / output blobs are one row of [rows][head_dim] per
 *     token with a token stride (ncnn cstep): packed QKV rows hold 3*H rows
 *     (q heads, k heads, v heads), attended / output rows hold H rows.
 */
#ifndef AWA_B200_H
#define AWA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* awa_stream_t; /* identical to cudaStream_t */
typedef struct awa_plan awa_plan;

#define AWA_OK 0
#define AWA_ERR_INVALID (-1)
#define AWA_ERR_CUDA (-2)
#define AWA_ERR_DEVICE (-3)
#define AWA_ERR_ALLOC (-100)

/* element types of blobs */
#define AWA_F32 0
#define AWA_BF16 1

/* attention arithmetic */
#define AWA_PREC_FP32 0 /* fp32 FFMA, fp32 accumulation, no TF32 (fp32 blocks) */
#define AWA_PREC_BF16 1 /* bf16 operands on tcgen05 tensor cores, fp32 accumulation (bf16 blocks) */

/* ParamDict ids 0-8 of the AWA layers (awa_layers.cpp:90-114, 872).
 * source_t/h/w == -1,-1,-1 means "take the grid from the runtime spec". */
typedef struct
{
    int source_t, source_h, source_w; /* ids 0,1,2: latent grid T x H x W */
    int windows_t, windows_h, windows_w; /* ids 3,4,5: target window COUNTS */
    int text_tokens;                  /* id 6 */
    int shifted;                      /* id 7: half-window shift (odd blocks) */
    int rope_dim;                     /* id 8: rotated features of Q/K, multiple of 6 (reference default 126) */
} awa_layer_params;

/* seedvr2::AwaRuntimeSpec (awa_layers.h:31-39). */
typedef struct
{
    int source_t, source_h, source_w, video_tokens;
} awa_runtime_spec;

/* seedvr2::AwaWindow (awa_layers.h:20-28): [t0,t1) x [h0,h1) x [w0,w1). */
typedef struct
{
    int t0, t1, h0, h1, w0, w1;
} awa_window;

typedef struct
{
    int source_t, source_h, source_w;
    int source_tokens;   /* N_v */
    int text_tokens;
    int window_count;    /* W */
    int sequence_tokens; /* S = sum of window lengths (video tokens + text tokens) */
    int max_window_length;
    int rope_dim;
    int shifted;
    int device;          /* CUDA device the plan's tables live on */
} awa_plan_info;

/* Replaces seedvr2::make_awa_windows (awa_layers.cpp:347-359, window rule
 * :53-88). Host only. Writes min(count, capacity) windows; returns the window
 * count, 0 for non-positive arguments. */
int awa_make_windows(int source_t, int source_h, int source_w, int windows_t, int windows_h, int windows_w,
                     int shifted, awa_window* out, int capacity);

/* Replaces the load_param of all four layers (awa_layers.cpp:382-417,
 * 599-636, 867-911, 1046-1060): builds the windows, index maps, cu_seqlens and
 * the RoPE table on the host and uploads them once to the CURRENT device.
 * spec may be NULL; it is required when params->source_* are -1 and must then
 * satisfy AwaRuntimeSpec::valid (awa_layers.cpp:340-345). rope_dim <= 0 means
 * 126. Returns -1 for what load_param rejects, -100 if an allocation fails. */
int awa_plan_create(const awa_layer_params* params, const awa_runtime_spec* spec, awa_plan** out_plan);
/* Same as awa_plan_create but builds the host tables only (no device, no
 * upload): for inspecting index maps on machines without a GPU. Every forward
 * entry point rejects such a plan with -1. */
int awa_plan_create_host(const awa_layer_params* params, const awa_runtime_spec* spec, awa_plan** out_plan);
void awa_plan_destroy(awa_plan* plan);
int awa_plan_get_info(const awa_plan* plan, awa_plan_info* info);

/* Host copies of the plan's index maps, for bit-exact checks. Each pointer may
 * be NULL; sizes are S, W+1, N_v and W*text_tokens ints. Windows: W entries. */
int awa_plan_get_maps(const awa_plan* plan, int* sequence_index, int* cu_seqlens, int* video_positions,
                      int* text_positions, awa_window* windows);

/* Replaces SeedVR2AWAPack::forward (awa_layers.cpp:419-458 CPU, 501-578 Vulkan).
 * packed: S rows of 3*H*head_dim (stride packed_token_stride >= 3*H*head_dim);
 * cu_seqlens: W+1 floats (the reference stores them as float). */
int awa_pack(const awa_plan* plan, int heads, int head_dim, int in_dtype, const void* video_qkv,
             int64_t video_token_stride, int64_t video_qkv_stride, const void* text_qkv, int64_t text_token_stride,
             int64_t text_qkv_stride, int out_dtype, void* packed, int64_t packed_token_stride, float* cu_seqlens,
             awa_stream_t stream);

/* Replaces SeedVR2MMRoPE::forward (awa_layers.cpp:913-953, 985-1025): rotates
 * the first rope_dim features of the Q and K rows in interleaved pairs;
 * V rows and the tail are copied. In fp32 the result is bit-identical to the
 * reference CPU forward. in and out may not alias. */
int awa_mmrope(const awa_plan* plan, int heads, int head_dim, int in_dtype, const void* packed_in,
               int64_t in_token_stride, int out_dtype, void* packed_out, int64_t out_token_stride,
               awa_stream_t stream);

/* Replaces SeedVR2WindowAttention::forward (awa_layers.cpp:1062-1120,
 * 1152-1234): per window and head, softmax(Q K^T / sqrt(d)) V over the
 * window's packed rows, no mask. Output: S rows of H*head_dim. */
int awa_window_attention(const awa_plan* plan, int precision, int heads, int head_dim, int in_dtype,
                         const void* packed, int64_t in_token_stride, int out_dtype, void* attended,
                         int64_t out_token_stride, awa_stream_t stream);

/* Replaces SeedVR2AWAUnpack::forward (awa_layers.cpp:638-689, 743-846):
 * video rows back to source order, text rows = mean over windows (sum of
 * x / W in window order, as the CPU forward). */
int awa_unpack(const awa_plan* plan, int heads, int head_dim, int in_dtype, const void* attended,
               int64_t in_token_stride, int out_dtype, void* video_out, int64_t video_token_stride,
               void* text_out, int64_t text_token_stride, awa_stream_t stream);

/* The whole chain Pack -> MMRoPE -> WindowAttention -> Unpack in one pass:
 * gathers each window's rows from the source QKV, rotates Q/K on the fly,
 * attends, scatters video rows to source order and reduces the text rows, so
 * no packed intermediate is written. Needs a workspace of
 * awa_forward_workspace_bytes(). Outputs equal the four-layer chain's. */
size_t awa_forward_workspace_bytes(const awa_plan* plan, int heads, int head_dim);
/* The workspace awa_forward needs for these precision and input dtype: the
 * above, plus, for fp32 QKV rows on the tensor-core path (AWA_PREC_BF16, a bf16
 * block fed the reference's promoted fp32 QKV, dit_precision.cpp:314-315), a
 * bf16 copy of the rows that one pass converts before the attention. */
size_t awa_forward_workspace_bytes_for(const awa_plan* plan, int precision, int in_dtype, int heads, int head_dim);
int awa_forward(const awa_plan* plan, int precision, int heads, int head_dim, int in_dtype, const void* video_qkv,
                int64_t video_token_stride, int64_t video_qkv_stride, const void* text_qkv,
                int64_t text_token_stride, int64_t text_qkv_stride, int out_dtype, void* video_out,
                int64_t video_token_stride_out, void* text_out, int64_t text_token_stride_out, void* workspace,
                size_t workspace_bytes, awa_stream_t stream);

/* awa_forward for Q/K rows that arrive rotated (awa_qkv_project_rotated with
 * this plan): the chain without the MMRoPE step -- Pack, WindowAttention,
 * Unpack. Same arguments, workspace and outputs as awa_forward. */
int awa_forward_prerotated(const awa_plan* plan, int precision, int heads, int head_dim, int in_dtype,
                           const void* video_qkv, int64_t video_token_stride, int64_t video_qkv_stride,
                           const void* text_qkv, int64_t text_token_stride, int64_t text_qkv_stride, int out_dtype,
                           void* video_out, int64_t video_token_stride_out, void* text_out,
                           int64_t text_token_stride_out, void* workspace, size_t workspace_bytes,
                           awa_stream_t stream);

/* awa_forward on HOST buffers -- the counterpart of the reference layers'
 * CPU forward, whose blobs are host Mats (awa_layers.cpp:419-458, 638-689,
 * 913-953, 1062-1120): video_qkv, text_qkv, video_out and text_out are host
 * pointers (pinned memory lets the copies run at the host link's rate and
 * overlap other streams); the call enqueues on `stream` the copies of the
 * QKV rows in, the fused forward and the copies of the outputs back, and
 * returns without waiting. device_workspace: awa_forward_host_workspace_bytes()
 * bytes of device memory (the device copies and awa_forward's workspace); the
 * host buffers must stay valid until the stream has done the work. */
size_t awa_forward_host_workspace_bytes(const awa_plan* plan, int precision, int in_dtype, int out_dtype, int heads,
                                        int head_dim);
int awa_forward_host(const awa_plan* plan, int precision, int heads, int head_dim, int in_dtype,
                     const void* video_qkv, int64_t video_token_stride, int64_t video_qkv_stride, const void* text_qkv,
                     int64_t text_token_stride, int64_t text_qkv_stride, int out_dtype, void* video_out,
                     int64_t video_token_stride_out, void* text_out, int64_t text_token_stride_out,
                     void* device_workspace, size_t workspace_bytes, awa_stream_t stream);

/* Size of the scratch that awa_forward_noalloc uses: 32 MiB of device memory
 * per GPU that loads this library, held until the process exits. */
#define AWA_NOALLOC_SCRATCH_BYTES (32u << 20)

/* awa_forward for callers that must not allocate device memory. Some hosts
 * cannot let a library call cudaMalloc: an inference server whose memory
 * manager reserves the whole GPU up front and owns every byte, a plugin whose
 * host framework hands out device memory only through its own allocator, or
 * a latency-bound pipeline that cannot afford the device-wide
 * synchronisation cudaMalloc/cudaFree cause. awa_forward needs the caller to
 * pass a workspace; this entry point instead uses a fixed scratch array that
 * the library holds in device memory (AWA_NOALLOC_SCRATCH_BYTES per GPU), and
 * it allocates nothing. No counterpart in the reference (its layers take
 * scratch from ncnn's workspace allocator).
 *   - Arguments, outputs and results are those of awa_forward, minus the
 *     workspace.
 *   - Limit: the layer's workspace (awa_forward_workspace_bytes) must fit in
 *     AWA_NOALLOC_SCRATCH_BYTES, e.g. 56 windows at 58 text tokens, 20 heads,
 *     head_dim 128. Larger layers get AWA_ERR_INVALID and a message; use
 *     awa_forward with a workspace for them. The check counts fp32 text
 *     partials, which the fp32 kernel writes; the tensor-core kernel writes
 *     them as bf16 and would need half, so on that path the limit is
 *     conservative by a factor of two.
 *   - Every call looks up the scratch's device address on the current device
 *     (which must be the plan's device), so a context created anew on the
 *     device (cudaDeviceReset) is picked up. The first call on a device loads
 *     the library's device code there: make it before any stream capture
 *     begins.
 *   - All calls on a GPU share the one scratch array, which keeps the last
 *     call's contents. Nothing in it needs to start at zero (each call writes
 *     every value it later reads), but calls that overlap on the GPU (other
 *     streams, other threads) race on it: order them on one stream or with
 *     events. */
int awa_forward_noalloc(const awa_plan* plan, int precision, int heads, int head_dim, int in_dtype,
                        const void* video_qkv, int64_t video_token_stride, int64_t video_qkv_stride,
                        const void* text_qkv, int64_t text_token_stride, int64_t text_qkv_stride, int out_dtype,
                        void* video_out, int64_t video_token_stride_out, void* text_out,
                        int64_t text_token_stride_out, awa_stream_t stream);

/* Window-parallel form of awa_forward for one rank of a multi-GPU group:
 * computes only the windows [window_begin, window_end) of the plan's window
 * order (every token of those windows is written to video_out; other rows
 * are left untouched) and writes the UNNORMALISED text partial sum
 * sum_{w in range} attended_text(w) to text_partial (fp32, text_tokens x H x
 * head_dim, dense). The caller all-reduces the partials and calls
 * awa_text_finalize. */
int awa_forward_windows(const awa_plan* plan, int precision, int heads, int head_dim, int window_begin,
                        int window_end, int in_dtype, const void* video_qkv, int64_t video_token_stride,
                        int64_t video_qkv_stride, const void* text_qkv, int64_t text_token_stride,
                        int64_t text_qkv_stride, int out_dtype, void* video_out, int64_t video_token_stride_out,
                        float* text_partial, void* workspace, size_t workspace_bytes, awa_stream_t stream);

/* text_out = text_sum / W (all windows of the plan), converted to out_dtype. */
int awa_text_finalize(const awa_plan* plan, int heads, int head_dim, const float* text_sum, int out_dtype,
                      void* text_out, int64_t text_token_stride, awa_stream_t stream);

/* Gathered-shard scatter for the multi-GPU path: rows of the packed video
 * shard layout (windows [window_begin, window_end) in plan order, video rows
 * only, dense H*head_dim rows) are copied to their source-order rows. */
int awa_scatter_video_shard(const awa_plan* plan, int heads, int head_dim, int window_begin, int window_end,
                            int dtype, const void* shard, void* video_out, int64_t video_token_stride,
                            awa_stream_t stream);
int awa_gather_video_shard(const awa_plan* plan, int heads, int head_dim, int window_begin, int window_end,
                           int dtype, const void* video, int64_t video_token_stride, void* shard,
                           awa_stream_t stream);
/* Number of video rows of windows [window_begin, window_end). */
int64_t awa_window_range_video_rows(const awa_plan* plan, int window_begin, int window_end);
/* Splits the plan's windows into `parts` contiguous ranges of near-equal
 * attention cost (sum of L^2); bounds receives parts+1 window indices. */
int awa_partition_windows(const awa_plan* plan, int parts, int* bounds);

/* ---- One layer split over the GPUs of a node.
 * Windows are independent (SeedVR2WindowAttention::forward,
 * awa_layers.cpp:1062-1120); the only coupling is the text mean
 * text += packed / window_count (SeedVR2AWAUnpack::forward :684-685). Each rank
 * computes a share of the layer and the ranks exchange the rest, so every rank
 * ends with the full outputs the ncnn boundary hands on:
 *   - window split: the windows sharing a (t-range, h-range) form a band --
 *     frames x whole grid lines -- and bands in (t, h) order are cut into runs
 *     of near-equal attention cost, one per rank, so a rank's video rows are a
 *     few contiguous token runs; the fp32 text partial sums are all-reduced
 *     (NCCL) and the video runs exchanged (below);
 *   - head split, with fewer bands than ranks or fewer than 4 windows per rank:
 *     each rank runs every window for a range of heads; the head slices of the
 *     video and text outputs are exchanged.
 * The video rows move either by NCCL all-gather (video_out in ordinary device
 * memory) or, when video_out lies in a buffer from awa_comm_alloc_shared, as
 * peer copies on the copy engines straight into every rank's copy, chunk by
 * chunk behind the attention. No kernel reads a peer's memory; nothing uses
 * TMA multicast. libnccl.so.2 is loaded on first use (inside a PyTorch
 * process: the NCCL torch loaded). */
typedef struct awa_comm awa_comm;

/* ncclGetUniqueId: rank 0 calls it and hands the bytes (128) to every rank. */
int awa_comm_unique_id(unsigned char* id, size_t capacity);
/* ncclCommInitRank on the current device; collective over the nranks ranks. */
int awa_comm_create(const unsigned char* id, size_t id_bytes, int nranks, int rank, awa_comm** out);
/* Uses the caller's own ncclComm_t (not destroyed by awa_comm_destroy). */
int awa_comm_wrap(void* nccl_comm, awa_comm** out);
/* Frees any shared buffer still held (without the barrier of
 * awa_comm_free_shared) and the communicator. */
void awa_comm_destroy(awa_comm* comm);
/* Collective: a device buffer of `bytes` (the same on every rank, else
 * AWA_ERR_INVALID) on every rank, each mapped into every other rank's address
 * space (CUDA IPC over NVLink). When video_out of awa_forward_sharded lies in
 * such a buffer -- at the same offset on every rank -- each rank's video rows
 * are pushed straight into every other rank's copy (no all-gather, staging or
 * scatter), behind an entry barrier so no rank overwrites rows another still
 * reads. *ptr is the local buffer (zeroed). */
int awa_comm_alloc_shared(awa_comm* comm, size_t bytes, void** ptr);
/* Collective: waits for every rank, unmaps and frees a shared buffer. */
int awa_comm_free_shared(awa_comm* comm, void* ptr);
/* How the direct mode moves a rank's video rows into the peers' copies:
 * AWA_PUSH_COPY_ENGINES -- one cudaMemcpyAsync per token run and peer on the
 * copy engines (one stream per peer), chunk by chunk behind the attention;
 * AWA_PUSH_KERNEL -- after one attention launch, an SM kernel loads each run
 * once and stores it into every peer over NVLink; AWA_PUSH_AUTO (default) --
 * the copy engines with one peer, the kernel with three or more. */
#define AWA_PUSH_AUTO 0
#define AWA_PUSH_COPY_ENGINES 1
#define AWA_PUSH_KERNEL 2
int awa_comm_set_push(awa_comm* comm, int mode);
int awa_comm_info(const awa_comm* comm, int* rank, int* nranks);
/* The split awa_forward_sharded uses for nranks ranks: *by_heads (0/1) and
 * nranks+1 bounds: head indices for a head split; for a window split the
 * prefix sums of the ranks' window counts. */
int awa_shard_split(const awa_plan* plan, int nranks, int heads, int* by_heads, int* bounds);
/* The windows (ascending plan indices) that `rank` computes in a window split
 * (every window for a head split): writes min(count, capacity), returns the
 * count. */
int awa_shard_windows(const awa_plan* plan, int nranks, int heads, int rank, int* windows, int capacity);
/* The video tokens `rank` computes in a window split, as runs of source-order
 * tokens: writes min(count, capacity) (first token, tokens) pairs to `runs`,
 * returns the count (a head split: one run of every token). These are the only
 * video QKV rows the rank's attention reads (besides the text rows), and the
 * rows of the output it writes: a caller can copy just these in from the host,
 * and out. */
int awa_shard_runs(const awa_plan* plan, int nranks, int heads, int rank, int64_t* runs, int capacity);
size_t awa_forward_sharded_workspace_bytes(const awa_plan* plan, int nranks, int heads, int head_dim, int out_dtype);
/* awa_forward over the ranks of `comm`: same arguments and outputs (on every
 * rank: inputs replicated, outputs complete), plus a workspace of
 * awa_forward_sharded_workspace_bytes(). Every rank must call it with the same
 * plan parameters; the collectives are enqueued on `stream`. */
int awa_forward_sharded(const awa_plan* plan, awa_comm* comm, int precision, int heads, int head_dim, int in_dtype,
                        const void* video_qkv, int64_t video_token_stride, int64_t video_qkv_stride,
                        const void* text_qkv, int64_t text_token_stride, int64_t text_qkv_stride, int out_dtype,
                        void* video_out, int64_t video_token_stride_out, void* text_out,
                        int64_t text_token_stride_out, void* workspace, size_t workspace_bytes, awa_stream_t stream);

/* The producer of the AWA input (the block's QKV projection with the per-head
 * RMSNorm of Q and K), on the tensor cores. Replaces, for one branch (video or
 * text) of a DiT block, proj_qkv + norm_q + norm_k of
 * tools/reference/dit_block.py:280-287 (ncnn: the block's Gemm, DitRMSNorm
 * src/dit/dit_precision.cpp:22-90 with shader dit_rmsnorm.comp, and
 * DitQKVConcat :95-142). out[t] = (RMSNorm_q(q heads), RMSNorm_k(k heads),
 * v heads) of bf16(x[t] W^T), the RMSNorm per head in fp32: y = x *
 * rsqrt(sum(x^2) / head_dim + eps) * gamma.
 *   x:   tokens rows of model_dim bf16, x_stride elements apart (16-byte rows)
 *   w:   the Linear weight as nn.Linear stores it: 3*heads*head_dim rows of
 *        model_dim bf16 ([out][in]), w_stride elements apart (16-byte rows)
 *   gamma_q, gamma_k: head_dim fp32 RMSNorm weights (device memory)
 *   out: tokens rows of 3*heads*head_dim out_dtype (AWA_BF16 or AWA_F32),
 *        out_stride elements apart (32-byte aligned rows): the rows
 *        awa_forward reads as video_qkv / text_qkv.
 * head_dim must be 128. The Q/K rows are rounded to out_dtype after the
 * RMSNorm (the reference keeps them in fp32 into its fp32 attention). */
int awa_qkv_project(int tokens, int model_dim, int heads, int head_dim, const void* x, int64_t x_stride,
                    const void* w, int64_t w_stride, const float* gamma_q, const float* gamma_k, float eps,
                    int out_dtype, void* out, int64_t out_stride, awa_stream_t stream);

/* Branches of a DiT block's QKV projection (awa_qkv_project_rotated). */
#define AWA_BRANCH_VIDEO 0
#define AWA_BRANCH_TEXT 1

/* awa_qkv_project with the layer's MMRoPE (SeedVR2MMRoPE, awa_layers.cpp:
 * 867-953) in its epilogue: after the RMSNorm, each Q and K head of token row
 * i is rotated in fp32 with the window-local coordinates the plan gives that
 * token -- (text_tokens + t - t0, h - h0, w - w0) of its window for the video
 * branch (tokens = the plan's video tokens, source order), (i, i, i) for the
 * text branch (tokens = the plan's text tokens) -- and rounded once to
 * out_dtype. The plan is the block's AWA layer plan (its shift decides the
 * windows). The rows then go to awa_forward_prerotated, which skips the
 * rotation. */
int awa_qkv_project_rotated(int tokens, int model_dim, int heads, int head_dim, const void* x, int64_t x_stride,
                            const void* w, int64_t w_stride, const float* gamma_q, const float* gamma_k, float eps,
                            const awa_plan* plan, int branch, int out_dtype, void* out, int64_t out_stride,
                            awa_stream_t stream);

/* The consumer of the AWA output, on the tensor cores: for one branch of a DiT
 * block, proj_out (a Linear with bias, tools/reference/dit_block.py:299), the
 * Ada "out" gate (FixedAdaBranch.forward mode "out", :187-190) and the
 * residual add (FixedDitBlock.forward :345-347):
 *   out[t][c] = residual[t][c] + bf16(x[t] W^T + bias)[c] * gate[c]
 * with (hidden * gate) and the sum each rounded to fp32, as the reference.
 *   x:        tokens rows of in_dim bf16 (the AWA output rows, heads*head_dim),
 *             x_stride elements apart (16-byte rows)
 *   w:        out_dim rows of in_dim bf16 ([out][in], nn.Linear's layout)
 *   bias, gate: out_dim fp32 (gate: the block's gate_a + gate_b for this step)
 *   residual: tokens rows of out_dim, residual_dtype (AWA_BF16 or AWA_F32),
 *             16-byte aligned rows (the block's input)
 *   out:      tokens rows of out_dim out_dtype, 32-byte aligned rows.
 * out_dim must be a multiple of 128. */
int awa_out_project(int tokens, int in_dim, int out_dim, const void* x, int64_t x_stride, const void* w,
                    int64_t w_stride, const float* bias, const float* gate, const void* residual,
                    int64_t residual_stride, int residual_dtype, int out_dtype, void* out, int64_t out_stride,
                    awa_stream_t stream);

/* Device-side status of the library on the current device: 0, or the code of
 * the first device check that failed since the last call (a bounded wait that
 * gave up). Synchronises the device. Clears the flag. */
int awa_device_status(void);

/* Self-test of the bounded waits that every wait in the library's kernels
 * uses (no counterpart in the reference). Launches one block of two warps that
 * wait on mbarriers nothing ever completes -- no copy, MMA or arrival is
 * issued, so nothing is in flight: the first warp with a limit of limit_us
 * microseconds (1..1000000), the second with a limit 1000 times longer, which
 * must end early on the abort flag the first warp raises when it gives up.
 * Synchronises the stream. *observed (host) gets bit 0 when the first wait
 * gave up, bit 1 when the second stopped on the abort; 3 is a pass. The give-up
 * sets the device status flag as a real one does (code 51), so the next
 * awa_device_status() returns AWA_ERR_DEVICE and clears it; the device stays
 * usable. */
int awa_selftest_bounded_wait(unsigned limit_us, int* observed, awa_stream_t stream);

/* Which attention kernel awa_forward would launch for these arguments:
 * 1 = tcgen05 (sm_100a tensor cores: AWA_PREC_BF16 with head_dim 128; fp32
 * QKV rows are first converted to bf16 in the workspace, see
 * awa_forward_workspace_bytes_for), 2 = fp32 SIMT (AWA_PREC_FP32, other head
 * sizes). awa_window_attention (packed rows) takes the tensor cores for bf16
 * packed rows only. */
int awa_attention_kernel_kind(const awa_plan* plan, int precision, int in_dtype, int heads, int head_dim);

/* Opt-in launch profiler (the counterpart of the reference's
 * PerformanceProfile, src/inference/performance_profile.h:75-227): while
 * enabled, every kernel the library launches is bracketed by CUDA events on
 * its own stream. awa_profile_collect synchronises those events and returns,
 * per kernel name, the launch count and total device milliseconds, formatted
 * as "profile name=<kernel> launches=<n> ms=<total>\n" lines. */
void awa_profile_enable(int enabled);
void awa_profile_reset(void);
int awa_profile_collect(char* buffer, size_t capacity);

const char* awa_last_error(void);
const char* awa_version(void);

#ifdef __cplusplus
}
#endif

#endif /* AWA_B200_H */
