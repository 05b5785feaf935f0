/*
 * awa_stack.h -- the AWA layers of a whole DiT block stack on one stream.
 *
 * The reference runs its 32 DiT blocks one ncnn Net at a time, submitting each
 * block's command buffer and waiting for it on the host before the next
 * (DitStackSession::run, src/dit/dit_stack.cpp:931-982, submit_and_wait at
 * :963), and switches the residual stream from fp32 to bf16 after the first 9
 * blocks (:519, :935-948). Each block's four AWA layers build their own
 * window tables in load_param.
 *
 * Here one awa_stack holds the plans of all blocks (blocks with identical
 * ParamDicts share one plan: a 32-block stack alternating shifted and
 * unshifted windows holds two) and one workspace, and runs every block's AWA
 * chain on the caller's stream with nothing that waits on the host. The
 * caller's own work around each block's attention (normalisation, the QKV
 * projection, proj_out, the MLP, the precision switch) is enqueued by a hook
 * the stack calls before and after each block, so the whole step can also be
 * captured once into a CUDA graph and replayed.
 */
#ifndef AWA_STACK_H
#define AWA_STACK_H

#include <stddef.h>
#include <stdint.h>

#include "awa_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct awa_stack awa_stack;
typedef struct awa_stack_graph awa_stack_graph;

#define AWA_STACK_BEFORE 0 /* hook stage: enqueue the block's work up to its QKV rows, fill the io */
#define AWA_STACK_AFTER 1  /* hook stage: enqueue the block's work after its attention output */

/* One block's AWA input and output, as awa_forward takes them. */
typedef struct
{
    int block;     /* set by the stack */
    int precision; /* set by the stack: AWA_PREC_FP32 in the fp32 prefix, AWA_PREC_BF16 after it */
    /* set by the hook at AWA_STACK_BEFORE (kept for AWA_STACK_AFTER): */
    int in_dtype;
    const void* video_qkv;
    int64_t video_token_stride, video_qkv_stride;
    const void* text_qkv;
    int64_t text_token_stride, text_qkv_stride;
    int out_dtype;
    void* video_out;
    int64_t video_out_stride;
    void* text_out;
    int64_t text_out_stride;
} awa_stack_io;

/* Called on the thread that runs the stack, in block order; enqueues work on
 * stream only (no host synchronisation, or a capture fails). Returns 0, or a
 * nonzero code that stops the run (awa_stack_run then returns AWA_ERR_INVALID). */
typedef int (*awa_stack_hook)(void* user, int stage, awa_stack_io* io, awa_stream_t stream);

/* Builds the stack on the CURRENT device: block_params[b] is block b's
 * ParamDict (e.g. awa_graph_find_chains of dit_block_<b>.ncnn.param), spec
 * the session's runtime spec (required when a grid is -1,-1,-1), fp32_blocks
 * the number of leading blocks computed in fp32 (9 for the reference's mixed
 * precision, blocks for its fp32 model, dit_stack.cpp:519). Allocates the
 * plans' tables and one workspace here; running allocates nothing. */
int awa_stack_create(const awa_layer_params* block_params, int blocks, const awa_runtime_spec* spec,
                     int fp32_blocks, int heads, int head_dim, awa_stack** out_stack);
void awa_stack_destroy(awa_stack* stack);
/* Number of distinct plans, workspace bytes; either pointer may be NULL. */
int awa_stack_get_info(const awa_stack* stack, int* plan_count, size_t* workspace_bytes);
/* The plan block b uses (owned by the stack), or NULL. */
const awa_plan* awa_stack_block_plan(const awa_stack* stack, int block);

/* Block b's AWA chain (awa_forward with the block's plan, precision and the
 * stack's workspace). Blocks share the workspace: run them in order on one
 * stream. */
int awa_stack_forward_block(awa_stack* stack, int block, const awa_stack_io* io, awa_stream_t stream);

/* All blocks in order on stream: hook(BEFORE), the block's AWA chain,
 * hook(AFTER). Returns the first nonzero status. */
int awa_stack_run(awa_stack* stack, awa_stack_hook hook, void* user, awa_stream_t stream);

/* awa_stack_run captured into a CUDA graph (thread-local capture on stream,
 * which must not be the legacy default stream) and instantiated; the hook's
 * work is captured with it. Run the stack once with awa_stack_run first, so
 * that first-use set-up (kernel attributes, the device status flag) happens
 * outside the capture. The graph replays the captured pointers: keep the
 * buffers the hook named alive and in place. */
int awa_stack_capture(awa_stack* stack, awa_stack_hook hook, void* user, awa_stream_t stream,
                      awa_stack_graph** out_graph);
int awa_stack_graph_launch(awa_stack_graph* graph, awa_stream_t stream);
void awa_stack_graph_destroy(awa_stack_graph* graph);

#ifdef __cplusplus
}
#endif

#endif /* AWA_STACK_H */
