// awa_noalloc.cu -- awa_forward for callers that must not allocate device
// memory (include/awa_b200.h: awa_forward_noalloc).
//
// Some hosts cannot let a library call cudaMalloc: a serving process whose
// memory manager has reserved the whole GPU, a plugin that may only use its
// host framework's allocator, a latency-bound pipeline that cannot take the
// device-wide synchronisation of cudaMalloc/cudaFree. For them the fused
// forward's one scratch buffer -- the fp32 per-window text partials that the
// attention kernel writes and the text reduction reads -- lives in a fixed
// array in device memory instead of a caller-provided workspace. Everything
// else is awa_forward itself.
#include "awa_b200.h"
#include "awa_internal.h"

#include <cuda_runtime.h>

#include <cstdio>

namespace
{

// The scratch: one copy per GPU that loads this library, kept until the
// process exits, shared by every call on that GPU. In host code this name is
// only a handle for cudaGetSymbolAddress, never a device address.
static __device__ __align__(256) unsigned char g_noalloc_scratch[AWA_NOALLOC_SCRATCH_BYTES];

// Device address of the scratch on the current device. Looked up on every
// call: the lookup is cheap once the module is loaded, and a context created
// anew on the device (after cudaDeviceReset) moves the array, so a cached
// address could go stale. The first lookup on a device loads the library's
// device code there, which must not happen inside a stream capture.
int scratch_address(void** out)
{
    void* p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (err != cudaSuccess || !p)
    {
        char message[256];
        std::snprintf(message, sizeof(message), "awa_forward_noalloc: cudaGetSymbolAddress failed: %s",
                      cudaGetErrorString(err));
        return awa::report_error(AWA_ERR_CUDA, message);
    }
    *out = p;
    return AWA_OK;
}

}  // namespace

extern "C" int awa_forward_noalloc(const awa_plan* plan, int precision, int heads, int head_dim, int in_dtype,
                                   const void* video_qkv, int64_t video_token_stride, int64_t video_qkv_stride,
                                   const void* text_qkv, int64_t text_token_stride, int64_t text_qkv_stride,
                                   int out_dtype, void* video_out, int64_t video_token_stride_out, void* text_out,
                                   int64_t text_token_stride_out, awa_stream_t stream)
{
    if (!plan || heads <= 0 || head_dim <= 0)
        return awa::report_error(AWA_ERR_INVALID, "awa_forward_noalloc: NULL plan or invalid heads / head_dim");
    const size_t need = awa_forward_workspace_bytes(plan, heads, head_dim);
    if (need == 0 || need > AWA_NOALLOC_SCRATCH_BYTES)
    {
        char message[256];
        std::snprintf(message, sizeof(message),
                      "awa_forward_noalloc: this layer needs %zu bytes of scratch, more than the %u bytes of "
                      "the library's fixed scratch; call awa_forward with a workspace instead",
                      need, (unsigned)AWA_NOALLOC_SCRATCH_BYTES);
        return awa::report_error(AWA_ERR_INVALID, message);
    }
    awa_plan_info info;
    int rc = awa_plan_get_info(plan, &info);
    if (rc)
        return rc;
    int device = -1;
    const cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess)
        return awa::report_error(AWA_ERR_CUDA, "awa_forward_noalloc: cudaGetDevice failed");
    if (info.device < 0 || device != info.device)
        return awa::report_error(AWA_ERR_INVALID,
                                 "awa_forward_noalloc: the plan's device must be the current device");
    void* scratch = nullptr;
    rc = scratch_address(&scratch);
    if (rc)
        return rc;
    // The attention kernel writes every text partial of the call before the
    // reduction reads it, so the scratch needs no clearing between calls.
    return awa_forward(plan, precision, heads, head_dim, in_dtype, video_qkv, video_token_stride, video_qkv_stride,
                       text_qkv, text_token_stride, text_qkv_stride, out_dtype, video_out, video_token_stride_out,
                       text_out, text_token_stride_out, scratch, AWA_NOALLOC_SCRATCH_BYTES, stream);
}
