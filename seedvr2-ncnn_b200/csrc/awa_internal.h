// awa_internal.h -- structures shared by the host plan (awa_plan.cpp) and the
// CUDA kernels (awa_copy_kernels.cu, awa_attn_simt.cu, awa_attn_tc.cu).
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

#include "awa_b200.h"

namespace awa
{

// One window of the plan, in make_windows order. Rows of a window are its
// video tokens in (t, h, w) row-major order, then the text tokens: the
// packed order of SeedVR2AWAPack (awa_layers.cpp:391-407).
struct WindowDesc
{
    int t0, h0, w0;  // clipped start (origin of the window-local RoPE coordinates)
    int nt, nh, nw;  // clipped extent
    int offset;      // first packed row (cu_seqlens[w])
    int video;       // nt * nh * nw
    int h0n, w0n;    // start of the unclipped (nominal-size) window: < h0, w0 only where clipped at 0
};

// Device tables of a plan (uploaded once by awa_plan_create).
struct PlanDevice
{
    const WindowDesc* windows = nullptr;
    const int* sequence_index = nullptr;   // [S]
    const int* cu_seqlens = nullptr;       // [W+1]
    const int* video_positions = nullptr;  // [N_v]
    const int* position_coords = nullptr;  // [S] short4 RoPE coordinates (t, h, w, 0) per packed row
    const float2* rope_table = nullptr;    // [max_coord][pairs_per_axis] (cos, sin)
    const uint2* rope_factors_bf16 = nullptr;  // same entries as bf16x2 words (cos, cos), (-sin, sin),
                                               // rows of pairs_per_axis rounded up to even
    int source_t = 0, source_h = 0, source_w = 0;
    int source_tokens = 0;
    int text_tokens = 0;
    int window_count = 0;
    int sequence_tokens = 0;
    int rope_dim = 0;
    int pairs_per_axis = 0;  // rope_dim / 6
    int max_coord = 0;
    int max_window_video = 0;  // most video rows of one window
    // Slab geometry of the tcgen05 kernel's fused path. A window's video rows
    // are fetched as boxes of tc_bhc x tc_bwc (h x w) tokens of one frame,
    // laid over the nominal window (tc_bh x tc_bw from (h0n, w0n)); every box
    // fills one 64-row key block (tc_rows rows used). Text rows follow in
    // blocks of 64 rows.
    int tc_bh = 0, tc_bw = 0;    // nominal window extent in h, w
    int tc_bhc = 0, tc_bwc = 0;  // box extent in h, w
    int tc_nhc = 0, tc_nwc = 0;  // boxes per frame along h, w
    int tc_rows = 0;             // tc_bhc * tc_bwc <= 64
    int tc_text_blocks = 0;      // ceil(text_tokens / 64)
};

enum DType : int
{
    kF32 = 0,
    kBF16 = 1
};

// Where an attention kernel reads its rows and writes its outputs.
//  packed mode: rows of window w are packed rows cu[w] .. cu[w+1]-1 of `qkv`
//               (q heads, k heads, v heads per row); outputs go to packed rows
//               of `out`. RoPE already applied (by the MMRoPE layer).
//  fused mode:  rows are gathered from the source QKV (video rows by window
//               geometry, text rows from the text QKV), Q/K are rotated on the
//               fly; video outputs go to source-order rows of `out`, text
//               outputs to `text_partial` [W][text][H][d] (fp32).
struct AttnArgs
{
    PlanDevice plan;
    int heads = 0;
    int head_dim = 0;
    float scale = 0.f;       // 1/sqrt(head_dim), as the reference computes it
    // packed mode
    const void* qkv = nullptr;
    int64_t qkv_token_stride = 0;
    // fused mode
    const void* video_qkv = nullptr;
    int64_t video_token_stride = 0, video_qkv_stride = 0;
    const void* text_qkv = nullptr;
    int64_t text_token_stride = 0, text_qkv_stride = 0;
    // outputs
    void* out = nullptr;
    int64_t out_token_stride = 0;
    // fused: [window - window_begin][text][H][d] text rows of each window, fp32
    // (SIMT kernel) or bf16 (tcgen05 kernel)
    float* text_partial = nullptr;
    // work list: (window, q tile) items (SIMT: 128-row tiles; tcgen05: pairs of
    // 128-row tiles), each taken for every head
    const int2* items = nullptr;
    int item_count = 0;
    int window_begin = 0;  // fused, sharded: first window of this launch
    int* error_flag = nullptr;
    int out_v8 = 0;  // tcgen05 kernel: output rows (and text partials) are 32-byte aligned
    int rotate = 1;  // fused: 1 = rotate Q/K as they are loaded, 0 = they arrive rotated (awa_qkv_project_rotated)
    // fused, a set of windows (multi-GPU): the text-partial slot of window w,
    // instead of w - window_begin
    const int* partial_slot = nullptr;
};

// Launchers (return a cudaError_t value as int).
int launch_pack(const PlanDevice& plan, int heads, int head_dim, int in_dtype, const void* video, int64_t vts,
                int64_t vqs, const void* text, int64_t tts, int64_t tqs, int out_dtype, void* packed, int64_t pts,
                float* cu_out, cudaStream_t stream);
int launch_mmrope(const PlanDevice& plan, int heads, int head_dim, int in_dtype, const void* in, int64_t its,
                  int out_dtype, void* out, int64_t ots, cudaStream_t stream);
int launch_unpack_video(const PlanDevice& plan, int heads, int head_dim, int in_dtype, const void* attended,
                        int64_t its, int out_dtype, void* video, int64_t vts, cudaStream_t stream);
// text_out[i] = mean over windows of src(w, i); src(w, i) is either packed row
// cu[w+1]-text+i of `attended` (packed != 0: the sum of src / divisor term by
// term in window order, as the reference's Unpack) or row (w*text+i) of a
// dense [W][text][H*d] array of in_dtype (the sum in window order, then /
// divisor).
// If divisor == 0 the sum is not divided and the result is written as fp32
// (partial sums).
int launch_text_reduce(const PlanDevice& plan, int heads, int head_dim, int packed, int in_dtype, const void* src,
                       int64_t src_token_stride, int window_begin, int window_end, float divisor, int out_dtype,
                       void* text_out, int64_t text_token_stride, cudaStream_t stream);
int launch_text_scale(int rows, int heads, int head_dim, const float* text_sum, float divisor, int out_dtype,
                      void* text_out, int64_t text_token_stride, cudaStream_t stream);
// fp32 QKV rows (token stride ts, q/k/v stride qs, `row` = H * d elements,
// a multiple of 8) -> dense bf16 rows [tokens][3][row], round to nearest even.
int launch_rows_to_bf16(const void* src, int64_t ts, int64_t qs, int tokens, int64_t row, void* dst,
                        cudaStream_t stream);
// The peers and byte runs of one push (launch_push_runs), in 16-byte units.
constexpr int kMaxPushPeers = 7;
constexpr int kMaxPushRuns = 96;
struct PushPeers
{
    uint4* ptr[kMaxPushPeers];
    int count;
};
struct PushRuns
{
    int64_t first[kMaxPushRuns];  // first 16-byte unit of each run
    int64_t count[kMaxPushRuns];  // units
    int n;
};
// Copies the runs of `local` into every peer at the same offsets (SM loads
// and NVLink stores), with a system-scope fence at the end of every thread.
int launch_push_runs(const void* local, const PushPeers& peers, const PushRuns& runs, cudaStream_t stream);
int launch_shard_copy(const PlanDevice& plan, int heads, int head_dim, int window_begin, int window_end, int dtype,
                      const void* src, int64_t src_stride, void* dst, int64_t dst_stride, int to_source,
                      cudaStream_t stream);

// Attention: packed != 0 selects packed mode. Template dispatch on dtypes.
int launch_attention_simt(const AttnArgs& args, int packed, int in_dtype, int out_dtype, cudaStream_t stream);
int launch_attention_tc(const AttnArgs& args, int packed, int in_dtype, int out_dtype, cudaStream_t stream);
// The bounded-wait self-test kernel (awa_selftest_bounded_wait).
int launch_wait_selftest(uint64_t limit_ns, int* error_flag, int* observed, cudaStream_t stream);
// x W^T with the per-head RMSNorm of Q and K (head_dim 128); arguments checked
// by the caller.
// rope_plan / rope_mode: 0 = no rotation; 1 = rows are the plan's video
// tokens, 2 = its text tokens: Q and K heads are rotated (MMRoPE, fp32, with
// each token's window-local coordinates) after the RMSNorm.
int launch_qkv_project(int tokens, int model_dim, int heads, const void* x, int64_t x_stride, const void* w,
                       int64_t w_stride, const float* gamma_q, const float* gamma_k, float eps, int out_dtype,
                       void* out, int64_t out_stride, cudaStream_t stream, const PlanDevice* rope_plan = nullptr,
                       int rope_mode = 0);
// out = resid + bf16(x W^T + bias) * gate per output channel (n_out % 128 == 0);
// arguments checked by the caller.
int launch_out_project(int tokens, int k_dim, int n_out, const void* x, int64_t x_stride, const void* w,
                       int64_t w_stride, const float* bias, const float* gate, const void* resid, int64_t resid_stride,
                       int resid_dtype, int out_dtype, void* out, int64_t out_stride, cudaStream_t stream);

int* device_error_flag();  // per-device flag in device memory

// The fused attention kernel alone over windows [window_begin, window_end):
// video rows into video_out, each window's text rows into the dense partials
// (window w at slot w - window_begin, of *partial_dtype: bf16 from the tcgen05
// kernel, fp32 from the SIMT kernel). partial_bytes bounds the slots.
int attention_range(const awa_plan* plan, int precision, int heads, int head_dim, int window_begin, int window_end,
                    int in_dtype, const void* video_qkv, int64_t video_token_stride, int64_t video_qkv_stride,
                    const void* text_qkv, int64_t text_token_stride, int64_t text_qkv_stride, int out_dtype,
                    void* video_out, int64_t video_token_stride_out, void* partials, size_t partial_bytes,
                    int* partial_dtype, cudaStream_t stream);
// attention_range over a set of windows (sorted, distinct): the text
// partials of the k-th window of the set go to slot k.
int attention_set(const awa_plan* plan, int precision, int heads, int head_dim, const int* windows, int count,
                  int in_dtype, const void* video_qkv, int64_t video_token_stride, int64_t video_qkv_stride,
                  const void* text_qkv, int64_t text_token_stride, int64_t text_qkv_stride, int out_dtype,
                  void* video_out, int64_t video_token_stride_out, void* partials, size_t partial_bytes,
                  int* partial_dtype, cudaStream_t stream);
// fp32 sum over windows [window_begin, window_end) of dense partials (slot
// w - window_begin), in window order, not divided.
int text_partial_sum(const awa_plan* plan, int heads, int head_dim, int partial_dtype, const void* partials,
                     int window_begin, int window_end, float* sum, cudaStream_t stream);
// Sets the calling thread's awa_last_error() text; returns code.
int report_error(int code, const char* message);

// Launch profiler: ProfileScope brackets one launch with events when enabled.
bool profiling_enabled();
void profile_record(const char* name, cudaEvent_t start, cudaEvent_t stop);
cudaEvent_t profile_event();
struct ProfileScope
{
    const char* name;
    cudaStream_t stream;
    cudaEvent_t start = nullptr;
    ProfileScope(const char* kernel, cudaStream_t s) : name(kernel), stream(s)
    {
        if (profiling_enabled())
        {
            start = profile_event();
            if (start)
                cudaEventRecord(start, stream);
        }
    }
    ~ProfileScope()
    {
        if (start)
        {
            cudaEvent_t stop = profile_event();
            if (stop)
            {
                cudaEventRecord(stop, stream);
                profile_record(name, start, stop);
            }
        }
    }
};

constexpr int kTcRowsPerTile = 128;   // query rows of one tcgen05 tile (a work item holds two)
constexpr int kSimtRowsPerTile = 128;  // query rows of one SIMT work item
constexpr int kMaxHeadDim = 128;

}  // namespace awa
