// awa_stack.cpp -- the AWA chains of a DiT block stack on one stream
// (counterpart of the block loop of DitStackSession::run,
// src/dit/dit_stack.cpp:931-982, without its per-block host wait).
#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "awa_b200.h"
#include "awa_internal.h"
#include "awa_stack.h"

struct awa_stack
{
    int blocks = 0;
    int fp32_blocks = 0;
    int heads = 0;
    int head_dim = 0;
    int device = 0;
    std::vector<awa_plan*> plans;
    std::vector<awa_layer_params> plan_params;
    std::vector<int> block_plan;
    void* workspace = nullptr;
    size_t workspace_bytes = 0;
};

struct awa_stack_graph
{
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
};

namespace
{

using awa::report_error;

int invalid(const std::string& message) { return report_error(AWA_ERR_INVALID, message.c_str()); }

int cuda_status(cudaError_t err, const char* what)
{
    if (err == cudaSuccess)
        return AWA_OK;
    const std::string message = std::string(what) + ": " + cudaGetErrorString(err);
    return report_error(err == cudaErrorMemoryAllocation ? AWA_ERR_ALLOC : AWA_ERR_CUDA, message.c_str());
}

bool same_params(const awa_layer_params& a, const awa_layer_params& b)
{
    const int rope_a = a.rope_dim > 0 ? a.rope_dim : 126, rope_b = b.rope_dim > 0 ? b.rope_dim : 126;
    return a.source_t == b.source_t && a.source_h == b.source_h && a.source_w == b.source_w &&
           a.windows_t == b.windows_t && a.windows_h == b.windows_h && a.windows_w == b.windows_w &&
           a.text_tokens == b.text_tokens && (a.shifted != 0) == (b.shifted != 0) && rope_a == rope_b;
}

int forward_block(awa_stack* s, int block, const awa_stack_io* io, cudaStream_t stream)
{
    const int precision = block < s->fp32_blocks ? AWA_PREC_FP32 : AWA_PREC_BF16;
    return awa_forward(s->plans[s->block_plan[block]], precision, s->heads, s->head_dim, io->in_dtype, io->video_qkv,
                       io->video_token_stride, io->video_qkv_stride, io->text_qkv, io->text_token_stride,
                       io->text_qkv_stride, io->out_dtype, io->video_out, io->video_out_stride, io->text_out,
                       io->text_out_stride, s->workspace, s->workspace_bytes, stream);
}

}  // namespace

extern "C" {

int awa_stack_create(const awa_layer_params* block_params, int blocks, const awa_runtime_spec* spec, int fp32_blocks,
                     int heads, int head_dim, awa_stack** out_stack)
{
    if (!out_stack)
        return invalid("awa_stack_create: null output");
    *out_stack = nullptr;
    if (!block_params || blocks <= 0 || fp32_blocks < 0 || fp32_blocks > blocks || heads <= 0 || head_dim <= 0)
        return invalid("awa_stack_create: invalid arguments (blocks > 0, 0 <= fp32_blocks <= blocks, heads and "
                       "head_dim > 0)");
    awa_stack* s = new awa_stack();
    s->blocks = blocks;
    s->fp32_blocks = fp32_blocks;
    s->heads = heads;
    s->head_dim = head_dim;
    int rc = cuda_status(cudaGetDevice(&s->device), "cudaGetDevice");
    for (int b = 0; rc == AWA_OK && b < blocks; b++)
    {
        int index = -1;
        for (size_t p = 0; p < s->plan_params.size(); p++)
            if (same_params(s->plan_params[p], block_params[b]))
                index = (int)p;
        if (index < 0)
        {
            awa_plan* plan = nullptr;
            rc = awa_plan_create(&block_params[b], spec, &plan);
            if (rc != AWA_OK)
                break;
            index = (int)s->plans.size();
            s->plans.push_back(plan);
            s->plan_params.push_back(block_params[b]);
        }
        s->block_plan.push_back(index);
    }
    for (size_t p = 0; rc == AWA_OK && p < s->plans.size(); p++)
        s->workspace_bytes = std::max(s->workspace_bytes, awa_forward_workspace_bytes(s->plans[p], heads, head_dim));
    if (rc == AWA_OK && s->workspace_bytes)
        rc = cuda_status(cudaMalloc(&s->workspace, s->workspace_bytes), "cudaMalloc(stack workspace)");
    // First use of the device status flag allocates it: do that here, not in a capture.
    if (rc == AWA_OK && !awa::device_error_flag())
        rc = invalid("awa_stack_create: device status flag unavailable");
    if (rc != AWA_OK)
    {
        awa_stack_destroy(s);
        return rc;
    }
    *out_stack = s;
    return AWA_OK;
}

void awa_stack_destroy(awa_stack* stack)
{
    if (!stack)
        return;
    for (awa_plan* plan : stack->plans)
        awa_plan_destroy(plan);
    if (stack->workspace)
        cudaFree(stack->workspace);
    delete stack;
}

int awa_stack_get_info(const awa_stack* stack, int* plan_count, size_t* workspace_bytes)
{
    if (!stack)
        return invalid("awa_stack_get_info: null stack");
    if (plan_count)
        *plan_count = (int)stack->plans.size();
    if (workspace_bytes)
        *workspace_bytes = stack->workspace_bytes;
    return AWA_OK;
}

const awa_plan* awa_stack_block_plan(const awa_stack* stack, int block)
{
    if (!stack || block < 0 || block >= stack->blocks)
        return nullptr;
    return stack->plans[stack->block_plan[block]];
}

int awa_stack_forward_block(awa_stack* stack, int block, const awa_stack_io* io, awa_stream_t stream)
{
    if (!stack || !io || block < 0 || block >= stack->blocks)
        return invalid("awa_stack_forward_block: invalid stack, io or block");
    return forward_block(stack, block, io, reinterpret_cast<cudaStream_t>(stream));
}

int awa_stack_run(awa_stack* stack, awa_stack_hook hook, void* user, awa_stream_t stream)
{
    if (!stack || !hook)
        return invalid("awa_stack_run: null stack or hook");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    for (int b = 0; b < stack->blocks; b++)
    {
        awa_stack_io io;
        std::memset(&io, 0, sizeof(io));
        io.block = b;
        io.precision = b < stack->fp32_blocks ? AWA_PREC_FP32 : AWA_PREC_BF16;
        int hook_rc = hook(user, AWA_STACK_BEFORE, &io, stream);
        if (hook_rc != 0)
            return invalid("awa_stack_run: hook returned " + std::to_string(hook_rc) + " before block " +
                           std::to_string(b));
        io.block = b;
        const int rc = forward_block(stack, b, &io, s);
        if (rc != AWA_OK)
            return rc;
        hook_rc = hook(user, AWA_STACK_AFTER, &io, stream);
        if (hook_rc != 0)
            return invalid("awa_stack_run: hook returned " + std::to_string(hook_rc) + " after block " +
                           std::to_string(b));
    }
    return AWA_OK;
}

int awa_stack_capture(awa_stack* stack, awa_stack_hook hook, void* user, awa_stream_t stream,
                      awa_stack_graph** out_graph)
{
    if (!out_graph)
        return invalid("awa_stack_capture: null output");
    *out_graph = nullptr;
    if (!stack || !hook || !stream)
        return invalid("awa_stack_capture: null stack, hook or stream (the legacy stream cannot be captured)");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int rc = cuda_status(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
    if (rc != AWA_OK)
        return rc;
    const int run_rc = awa_stack_run(stack, hook, user, stream);
    cudaGraph_t graph = nullptr;
    const cudaError_t end_err = cudaStreamEndCapture(s, &graph);  // always close the capture
    if (run_rc != AWA_OK)
    {
        if (graph)
            cudaGraphDestroy(graph);
        return run_rc;
    }
    rc = cuda_status(end_err, "cudaStreamEndCapture");
    if (rc != AWA_OK)
    {
        if (graph)
            cudaGraphDestroy(graph);
        return rc;
    }
    awa_stack_graph* g = new awa_stack_graph();
    g->graph = graph;
    rc = cuda_status(cudaGraphInstantiate(&g->exec, graph, 0), "cudaGraphInstantiate");
    if (rc != AWA_OK)
    {
        awa_stack_graph_destroy(g);
        return rc;
    }
    *out_graph = g;
    return AWA_OK;
}

int awa_stack_graph_launch(awa_stack_graph* graph, awa_stream_t stream)
{
    if (!graph || !graph->exec)
        return invalid("awa_stack_graph_launch: null graph");
    return cuda_status(cudaGraphLaunch(graph->exec, reinterpret_cast<cudaStream_t>(stream)), "cudaGraphLaunch");
}

void awa_stack_graph_destroy(awa_stack_graph* graph)
{
    if (!graph)
        return;
    if (graph->exec)
        cudaGraphExecDestroy(graph->exec);
    if (graph->graph)
        cudaGraphDestroy(graph->graph);
    delete graph;
}

}  // extern "C"
