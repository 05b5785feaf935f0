// awa_host.cpp -- the fused AWA forward on host buffers (include/awa_b200.h:
// awa_forward_host), the counterpart of the reference layers' CPU forward
// (Mat blobs in host memory, awa_layers.cpp:419-458, 913-953, 1062-1120,
// 638-689): the QKV rows are copied in, the chain runs on the GPU, the outputs
// are copied back, all enqueued on the caller's stream.
#include "awa_b200.h"
#include "awa_internal.h"

#include <cstdarg>
#include <cstdio>

#include <cuda_runtime.h>

namespace
{

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

size_t a256(size_t v)
{
    return (v + 255) & ~(size_t)255;
}

size_t dsize(int dtype)
{
    return dtype == AWA_BF16 ? 2 : 4;
}

struct HostLayout
{
    size_t video_in = 0, text_in = 0, video_out = 0, text_out = 0, forward = 0, total = 0;
};

HostLayout host_layout(const awa_plan_info& info, const awa_plan* plan, int precision, int in_dtype, int out_dtype,
                       int heads, int head_dim)
{
    HostLayout l;
    const size_t row = (size_t)heads * head_dim;
    size_t off = 0;
    l.video_in = off;
    off += a256((size_t)info.source_tokens * 3 * row * dsize(in_dtype));
    l.text_in = off;
    off += a256((size_t)info.text_tokens * 3 * row * dsize(in_dtype));
    l.video_out = off;
    off += a256((size_t)info.source_tokens * row * dsize(out_dtype));
    l.text_out = off;
    off += a256((size_t)info.text_tokens * row * dsize(out_dtype));
    l.forward = off;
    off += a256(awa_forward_workspace_bytes_for(plan, precision, in_dtype, heads, head_dim));
    l.total = off;
    return l;
}

// QKV rows of a strided host blob (token stride ts, q/k/v stride qs, in
// elements) -> a dense device array [tokens][3][H*d]: one copy when the blob
// is dense, else one pitched copy per q/k/v segment.
cudaError_t copy_qkv_in(void* dense, const void* blob, int64_t ts, int64_t qs, int tokens, size_t row_bytes, size_t es,
                        cudaStream_t st)
{
    if ((size_t)ts * es == 3 * row_bytes && (size_t)qs * es == row_bytes)
        return cudaMemcpyAsync(dense, blob, (size_t)tokens * 3 * row_bytes, cudaMemcpyHostToDevice, st);
    for (int q = 0; q < 3; q++)
    {
        const cudaError_t e = cudaMemcpy2DAsync(static_cast<unsigned char*>(dense) + q * row_bytes, 3 * row_bytes,
                                                static_cast<const unsigned char*>(blob) + q * qs * es, ts * es,
                                                row_bytes, tokens, cudaMemcpyHostToDevice, st);
        if (e != cudaSuccess)
            return e;
    }
    return cudaSuccess;
}

}  // namespace

extern "C" {

size_t awa_forward_host_workspace_bytes(const awa_plan* plan, int precision, int in_dtype, int out_dtype, int heads,
                                        int head_dim)
{
    awa_plan_info info;
    if (!plan || heads <= 0 || head_dim <= 0 || awa_plan_get_info(plan, &info) != AWA_OK)
        return 0;
    return host_layout(info, plan, precision, in_dtype, out_dtype, heads, head_dim).total;
}

int awa_forward_host(const awa_plan* plan, int precision, int heads, int head_dim, int in_dtype,
                     const void* video_qkv, int64_t video_token_stride, int64_t video_qkv_stride, const void* text_qkv,
                     int64_t text_token_stride, int64_t text_qkv_stride, int out_dtype, void* video_out,
                     int64_t video_token_stride_out, void* text_out, int64_t text_token_stride_out,
                     void* device_workspace, size_t workspace_bytes, awa_stream_t stream)
{
    awa_plan_info info;
    if (!plan || awa_plan_get_info(plan, &info) != AWA_OK || heads <= 0 || head_dim <= 0 || !video_qkv ||
        !text_qkv || !video_out || !text_out || !device_workspace ||
        (in_dtype != AWA_F32 && in_dtype != AWA_BF16) || (out_dtype != AWA_F32 && out_dtype != AWA_BF16))
        return fail(AWA_ERR_INVALID, "awa_forward_host: invalid arguments");
    const int64_t row = (int64_t)heads * head_dim;
    if (video_token_stride < row || video_qkv_stride < row || text_token_stride < row || text_qkv_stride < row ||
        video_token_stride_out < row || text_token_stride_out < row)
        return fail(AWA_ERR_INVALID, "awa_forward_host: strides smaller than a row");
    const HostLayout l = host_layout(info, plan, precision, in_dtype, out_dtype, heads, head_dim);
    if (workspace_bytes < l.total)
        return fail(AWA_ERR_INVALID, "awa_forward_host: device workspace of %zu bytes needed, %zu given", l.total,
                    workspace_bytes);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    unsigned char* ws = static_cast<unsigned char*>(device_workspace);
    const size_t ies = dsize(in_dtype), oes = dsize(out_dtype);
    cudaError_t e = copy_qkv_in(ws + l.video_in, video_qkv, video_token_stride, video_qkv_stride, info.source_tokens,
                                row * ies, ies, st);
    if (e == cudaSuccess)
        e = copy_qkv_in(ws + l.text_in, text_qkv, text_token_stride, text_qkv_stride, info.text_tokens, row * ies, ies,
                        st);
    if (e != cudaSuccess)
        return fail(AWA_ERR_CUDA, "awa_forward_host: copy in: %s", cudaGetErrorString(e));
    int rc = awa_forward(plan, precision, heads, head_dim, in_dtype, ws + l.video_in, 3 * row, row, ws + l.text_in,
                         3 * row, row, out_dtype, ws + l.video_out, row, ws + l.text_out, row, ws + l.forward,
                         l.total - l.forward, stream);
    if (rc)
        return rc;
    e = cudaMemcpy2DAsync(video_out, video_token_stride_out * oes, ws + l.video_out, row * oes, row * oes,
                          info.source_tokens, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess)
        e = cudaMemcpy2DAsync(text_out, text_token_stride_out * oes, ws + l.text_out, row * oes, row * oes,
                              info.text_tokens, cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess)
        return fail(AWA_ERR_CUDA, "awa_forward_host: copy out: %s", cudaGetErrorString(e));
    return AWA_OK;
}

}  // extern "C"
