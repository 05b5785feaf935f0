// awa_layers.cpp -- ncnn layer classes of SeedVR2 AWA over the B200 C ABI.
// Interface contract: HGinkgo/SeedVR2-ncnn src/awa/awa_layers.{h,cpp}
// (constructor flags :363-373, :581-590, :849-858, :1028-1037; load_param and
// forward of each layer; registration :1237-1291).
#include "awa_layers.h"

#include <cstdio>
#include <cstring>
#include <limits>

#include <cuda_runtime.h>

#include "net.h"

namespace
{

// ncnn return codes (0 / -1 / -100); CUDA-side failures read as -1 like the
// reference's Vulkan path does, with the library's message on stderr.
int to_ncnn_status(int rc, const char* layer)
{
    if (rc == AWA_OK)
        return 0;
    std::fprintf(stderr, "%s: %s\n", layer, awa_last_error());
    return rc == AWA_ERR_ALLOC ? -100 : -1;
}

struct QkvLayout
{
    int heads = 0;
    int head_dim = 0;
    int64_t token_stride = 0;
    int64_t qkv_stride = 0;
};

// The QKV blob encodings of describe_qkv_layout (awa_layers.cpp:124-170),
// for any blob type with ncnn Mat geometry: (w=d, h=3H, c=N), (w=d, h=H,
// c=3N), (dims 4: w=d, h=H, d=3, c=N) and, in NCNN_BATCH builds, (w=d, h=H,
// c=3, n=N) with one token per batch item.
template <typename Blob>
bool describe_qkv(const Blob& b, int tokens, QkvLayout& layout)
{
    if (b.w <= 0 || b.h <= 0)
        return false;
    layout.head_dim = b.w;
    if (b.dims == 3)
    {
        if (b.h % 3 == 0 && b.c == tokens)
        {
            layout.heads = b.h / 3;
            layout.token_stride = (int64_t)b.cstep;
            layout.qkv_stride = (int64_t)layout.heads * b.w;
        }
        else if (b.c == tokens * 3)
        {
            layout.heads = b.h;
            layout.token_stride = (int64_t)b.cstep;
            layout.qkv_stride = (int64_t)tokens * (int64_t)b.cstep;
        }
#if NCNN_BATCH
        else if (b.c == 3 && b.n == tokens)
        {
            layout.heads = b.h;
            layout.token_stride = (int64_t)b.nstep;
            layout.qkv_stride = (int64_t)b.cstep;
        }
#endif
        else
            return false;
    }
    else if (b.dims == 4)
    {
        if (b.d != 3 || b.c != tokens)
            return false;
        layout.heads = b.h;
        layout.token_stride = (int64_t)b.cstep;
        layout.qkv_stride = (int64_t)b.h * b.w;
    }
    else
        return false;
    return layout.heads > 0;
}

bool describe(const ncnn::Mat& m, int tokens, QkvLayout& layout)
{
    return m.elempack == 1 && (m.elemsize == 4u || m.elemsize == 2u) && describe_qkv(m, tokens, layout);
}

bool describe(const seedvr2::CudaBlob& b, int tokens, QkvLayout& layout)
{
    return (b.elemsize == 4u || b.elemsize == 2u) && describe_qkv(b, tokens, layout);
}

int dtype_of(size_t elemsize)
{
    return elemsize == 2u ? AWA_BF16 : AWA_F32;
}

// Bytes from a blob's first element to the end of its storage.
template <typename Blob>
size_t blob_bytes(const Blob& m)
{
    const size_t one = m.dims >= 3 ? m.cstep * m.c : (size_t)m.w * m.h;
    return (m.n > 1 ? m.nstep * (size_t)(m.n - 1) + one : one) * m.elemsize;
}

size_t mat_bytes(const ncnn::Mat& m)
{
    return blob_bytes(m);
}

size_t align16(size_t bytes)
{
    return (bytes + 15) & ~(size_t)15;
}

}  // namespace

namespace seedvr2
{

bool AwaRuntimeSpec::valid() const
{
    const long long tokens = static_cast<long long>(source_t) * source_h * source_w;
    return source_t > 0 && source_h > 0 && source_w > 0 && video_tokens > 0 && tokens == video_tokens &&
           tokens <= std::numeric_limits<int>::max();
}

std::vector<AwaWindow> make_awa_windows(int source_t, int source_h, int source_w, int windows_t, int windows_h,
                                        int windows_w, bool shifted)
{
    const int count =
        awa_make_windows(source_t, source_h, source_w, windows_t, windows_h, windows_w, shifted ? 1 : 0, nullptr, 0);
    std::vector<awa_window> raw(count > 0 ? count : 0);
    awa_make_windows(source_t, source_h, source_w, windows_t, windows_h, windows_w, shifted ? 1 : 0, raw.data(), count);
    std::vector<AwaWindow> out;
    out.reserve(raw.size());
    for (const awa_window& w : raw)
    {
        AwaWindow win;
        win.t0 = w.t0;
        win.t1 = w.t1;
        win.h0 = w.h0;
        win.h1 = w.h1;
        win.w0 = w.w0;
        win.w1 = w.w1;
        out.push_back(win);
    }
    return out;
}

int cuda_blob_create(CudaBlob& blob, int dims, int w, int h, int d, int c, size_t elemsize, int n)
{
    cuda_blob_free(blob);
    blob.dims = dims;
    blob.w = w;
    blob.h = h;
    blob.d = d;
    blob.c = c;
    blob.n = n;
    blob.elemsize = elemsize;
    blob.cstep = dims >= 3 ? align16((size_t)w * h * d * elemsize) / elemsize : (size_t)w * h;
    blob.nstep = blob.cstep * (dims >= 3 ? c : 1);
    if (n > 1)
        blob.nstep = ((blob.nstep * elemsize + 4095) & ~(size_t)4095) / elemsize;
    const size_t bytes = align16(blob.nstep * (size_t)n * elemsize);
    if (bytes == 0 || cudaMalloc(&blob.data, bytes) != cudaSuccess)
    {
        blob.data = nullptr;
        return -100;
    }
    blob.owned = true;
    return 0;
}

void cuda_blob_free(CudaBlob& blob)
{
    if (blob.owned && blob.data)
        cudaFree(blob.data);
    blob.data = nullptr;
    blob.owned = false;
}

AwaLayerBase::AwaLayerBase()
{
    one_blob_only = false;
    support_inplace = false;
    support_vulkan = false;  // this build's device path is forward_cuda
    support_packing = false;
    support_any_packing = false;
    support_vulkan_packing = false;
    support_vulkan_any_packing = false;
}

AwaLayerBase::AwaLayerBase(const AwaRuntimeSpec& runtime_spec) : AwaLayerBase()
{
    has_runtime_spec_ = true;
    runtime_spec_ = runtime_spec;
}

AwaLayerBase::~AwaLayerBase()
{
    awa_plan_destroy(plan_);
    for (void* p : staging_)
        if (p)
            cudaFree(p);
}

// load_common (awa_layers.cpp:90-114) + the per-layer maps, built once by the plan.
int AwaLayerBase::load_common_params(const ncnn::ParamDict& pd, int rope_dim)
{
    awa_layer_params params;
    params.source_t = pd.get(0, 0);
    params.source_h = pd.get(1, 0);
    params.source_w = pd.get(2, 0);
    params.windows_t = pd.get(3, 0);
    params.windows_h = pd.get(4, 0);
    params.windows_w = pd.get(5, 0);
    params.text_tokens = pd.get(6, 0);
    params.shifted = pd.get(7, 0) != 0;
    params.rope_dim = rope_dim;
    awa_runtime_spec spec;
    spec.source_t = runtime_spec_.source_t;
    spec.source_h = runtime_spec_.source_h;
    spec.source_w = runtime_spec_.source_w;
    spec.video_tokens = runtime_spec_.video_tokens;
    if (params.source_t == -1 && params.source_h == -1 && params.source_w == -1 &&
        (!has_runtime_spec_ || !runtime_spec_.valid()))
        return -1;
    awa_plan_destroy(plan_);
    plan_ = nullptr;
    const int rc = awa_plan_create(&params, has_runtime_spec_ ? &spec : nullptr, &plan_);
    if (rc != AWA_OK)
        return rc == AWA_ERR_ALLOC ? -100 : -1;
    awa_plan_get_info(plan_, &info_);
    return 0;
}

void* AwaLayerBase::staging(int slot, size_t bytes) const
{
    if (staging_bytes_[slot] < bytes)
    {
        if (staging_[slot])
            cudaFree(staging_[slot]);
        staging_[slot] = nullptr;
        staging_bytes_[slot] = 0;
        if (cudaMalloc(&staging_[slot], bytes) != cudaSuccess)
        {
            staging_[slot] = nullptr;
            return nullptr;
        }
        staging_bytes_[slot] = bytes;
    }
    return staging_[slot];
}

} // namespace seedvr2

using seedvr2::CudaBlob;
using seedvr2::CudaOption;

namespace
{

bool bf16_blocks(const ncnn::Option& opt)
{
    return opt.use_bf16_storage || opt.use_bf16_packed;  // awa_bf16_io, awa_layers.cpp:184-187
}

cudaError_t upload(void* dst, const ncnn::Mat& m)
{
    return cudaMemcpyAsync(dst, m.data, mat_bytes(m), cudaMemcpyHostToDevice, 0);
}

cudaError_t download(ncnn::Mat& m, const void* src)
{
    return cudaMemcpyAsync(m.data, src, mat_bytes(m), cudaMemcpyDeviceToHost, 0);
}

int finish(cudaError_t err, int rc, const char* layer)
{
    if (rc != AWA_OK)
        return to_ncnn_status(rc, layer);
    if (err == cudaSuccess)
        err = cudaStreamSynchronize(0);
    if (err != cudaSuccess)
    {
        std::fprintf(stderr, "%s: %s\n", layer, cudaGetErrorString(err));
        return -1;
    }
    return 0;
}

}  // namespace

// ------------------------------------------------------------------ Pack
SeedVR2AWAPack::SeedVR2AWAPack()
{
    support_batch = true;
}

SeedVR2AWAPack::SeedVR2AWAPack(const seedvr2::AwaRuntimeSpec& runtime_spec) : seedvr2::AwaLayerBase(runtime_spec)
{
    support_batch = true;
}

int SeedVR2AWAPack::load_param(const ncnn::ParamDict& pd)
{
    return load_common_params(pd, 126);
}

int SeedVR2AWAPack::forward(const std::vector<ncnn::Mat>& bottom_blobs, std::vector<ncnn::Mat>& top_blobs,
                            const ncnn::Option& opt) const
{
    if (bottom_blobs.size() != 2 || !plan_)
        return -1;
    const ncnn::Mat& video = bottom_blobs[0];
    const ncnn::Mat& text = bottom_blobs[1];
    QkvLayout vl, tl;
    if (!describe(video, info_.source_tokens, vl) || !describe(text, info_.text_tokens, tl) || vl.heads != tl.heads ||
        vl.head_dim != tl.head_dim || video.elemsize != text.elemsize)
        return -1;
    const size_t out_elem = bf16_blocks(opt) ? 2u : 4u;
    top_blobs.resize(2);
    top_blobs[0].create(vl.head_dim, 3 * vl.heads, info_.sequence_tokens, out_elem, opt.blob_allocator);
    top_blobs[1].create(info_.window_count + 1, 4u, opt.blob_allocator);
    if (top_blobs[0].empty() || top_blobs[1].empty())
        return -100;
    std::lock_guard<std::mutex> lock(mutex_);
    void* dv = staging(0, mat_bytes(video));
    void* dt = staging(1, mat_bytes(text));
    void* dp = staging(2, mat_bytes(top_blobs[0]));
    void* dc = staging(3, mat_bytes(top_blobs[1]));
    if (!dv || !dt || !dp || !dc)
        return -100;
    cudaError_t err = upload(dv, video);
    if (err == cudaSuccess)
        err = upload(dt, text);
    int rc = AWA_OK;
    if (err == cudaSuccess)
        rc = awa_pack(plan_, vl.heads, vl.head_dim, dtype_of(video.elemsize), dv, vl.token_stride, vl.qkv_stride, dt,
                      tl.token_stride, tl.qkv_stride, dtype_of(out_elem), dp, (int64_t)top_blobs[0].cstep,
                      static_cast<float*>(dc), nullptr);
    if (err == cudaSuccess && rc == AWA_OK)
        err = download(top_blobs[0], dp);
    if (err == cudaSuccess && rc == AWA_OK)
        err = download(top_blobs[1], dc);
    return finish(err, rc, "SeedVR2AWAPack");
}

int SeedVR2AWAPack::forward_cuda(const std::vector<CudaBlob>& bottom_blobs, std::vector<CudaBlob>& top_blobs,
                                 const CudaOption& opt) const
{
    if (bottom_blobs.size() != 2 || !plan_)
        return -1;
    const CudaBlob& video = bottom_blobs[0];
    const CudaBlob& text = bottom_blobs[1];
    QkvLayout vl, tl;
    if (!describe(video, info_.source_tokens, vl) || !describe(text, info_.text_tokens, tl) || vl.heads != tl.heads ||
        vl.head_dim != tl.head_dim || video.elemsize != text.elemsize)
        return -1;
    const size_t out_elem = opt.use_bf16_storage ? 2u : 4u;
    top_blobs.resize(2);
    if (seedvr2::cuda_blob_create(top_blobs[0], 3, vl.head_dim, 3 * vl.heads, 1, info_.sequence_tokens, out_elem) ||
        seedvr2::cuda_blob_create(top_blobs[1], 1, info_.window_count + 1, 1, 1, 1, 4u))
        return -100;
    return to_ncnn_status(awa_pack(plan_, vl.heads, vl.head_dim, dtype_of(video.elemsize), video.data, vl.token_stride,
                                   vl.qkv_stride, text.data, tl.token_stride, tl.qkv_stride, dtype_of(out_elem),
                                   top_blobs[0].data, (int64_t)top_blobs[0].cstep, static_cast<float*>(top_blobs[1].data),
                                   opt.stream),
                          "SeedVR2AWAPack");
}

// ------------------------------------------------------------------ MMRoPE
SeedVR2MMRoPE::SeedVR2MMRoPE() {}

SeedVR2MMRoPE::SeedVR2MMRoPE(const seedvr2::AwaRuntimeSpec& runtime_spec) : seedvr2::AwaLayerBase(runtime_spec) {}

int SeedVR2MMRoPE::load_param(const ncnn::ParamDict& pd)
{
    rope_dim_ = pd.get(8, 126);
    if (rope_dim_ <= 0 || rope_dim_ % 6 != 0)  // awa_layers.cpp:872-874
        return -1;
    return load_common_params(pd, rope_dim_);
}

int SeedVR2MMRoPE::forward(const std::vector<ncnn::Mat>& bottom_blobs, std::vector<ncnn::Mat>& top_blobs,
                           const ncnn::Option& opt) const
{
    if (bottom_blobs.size() != 1 || !plan_)
        return -1;
    const ncnn::Mat& input = bottom_blobs[0];
    if (input.dims != 3 || input.elempack != 1 || (input.elemsize != 4u && input.elemsize != 2u) ||
        input.w < rope_dim_ || input.h <= 0 || input.h % 3 != 0 || input.c != info_.sequence_tokens)
        return -1;
    const size_t out_elem = bf16_blocks(opt) ? 2u : 4u;
    top_blobs.resize(1);
    top_blobs[0].create(input.w, input.h, input.c, out_elem, opt.blob_allocator);
    if (top_blobs[0].empty())
        return -100;
    std::lock_guard<std::mutex> lock(mutex_);
    void* din = staging(0, mat_bytes(input));
    void* dout = staging(1, mat_bytes(top_blobs[0]));
    if (!din || !dout)
        return -100;
    cudaError_t err = upload(din, input);
    int rc = AWA_OK;
    if (err == cudaSuccess)
        rc = awa_mmrope(plan_, input.h / 3, input.w, dtype_of(input.elemsize), din, (int64_t)input.cstep,
                        dtype_of(out_elem), dout, (int64_t)top_blobs[0].cstep, nullptr);
    if (err == cudaSuccess && rc == AWA_OK)
        err = download(top_blobs[0], dout);
    return finish(err, rc, "SeedVR2MMRoPE");
}

int SeedVR2MMRoPE::forward_cuda(const std::vector<CudaBlob>& bottom_blobs, std::vector<CudaBlob>& top_blobs,
                                const CudaOption& opt) const
{
    if (bottom_blobs.size() != 1 || !plan_)
        return -1;
    const CudaBlob& input = bottom_blobs[0];
    if (input.dims != 3 || (input.elemsize != 4u && input.elemsize != 2u) || input.w < rope_dim_ || input.h <= 0 ||
        input.h % 3 != 0 || input.c != info_.sequence_tokens)
        return -1;
    const size_t out_elem = opt.use_bf16_storage ? 2u : 4u;
    top_blobs.resize(1);
    if (seedvr2::cuda_blob_create(top_blobs[0], 3, input.w, input.h, 1, input.c, out_elem))
        return -100;
    return to_ncnn_status(awa_mmrope(plan_, input.h / 3, input.w, dtype_of(input.elemsize), input.data,
                                     (int64_t)input.cstep, dtype_of(out_elem), top_blobs[0].data,
                                     (int64_t)top_blobs[0].cstep, opt.stream),
                          "SeedVR2MMRoPE");
}

// ------------------------------------------------------------------ WindowAttention
SeedVR2WindowAttention::SeedVR2WindowAttention() {}

SeedVR2WindowAttention::SeedVR2WindowAttention(const seedvr2::AwaRuntimeSpec& runtime_spec)
    : seedvr2::AwaLayerBase(runtime_spec)
{
}

int SeedVR2WindowAttention::load_param(const ncnn::ParamDict& pd)
{
    return load_common_params(pd, 126);
}

int SeedVR2WindowAttention::forward(const std::vector<ncnn::Mat>& bottom_blobs, std::vector<ncnn::Mat>& top_blobs,
                                    const ncnn::Option& opt) const
{
    if (bottom_blobs.size() != 1 || !plan_)
        return -1;
    const ncnn::Mat& input = bottom_blobs[0];
    if (input.dims != 3 || input.elempack != 1 || (input.elemsize != 4u && input.elemsize != 2u) || input.w <= 0 ||
        input.h <= 0 || input.h % 3 != 0 || input.c != info_.sequence_tokens)
        return -1;
    const bool bf16 = bf16_blocks(opt);
    const size_t out_elem = bf16 ? 2u : 4u;
    const int heads = input.h / 3;
    top_blobs.resize(1);
    top_blobs[0].create(input.w, heads, info_.sequence_tokens, out_elem, opt.blob_allocator);
    if (top_blobs[0].empty())
        return -100;
    std::lock_guard<std::mutex> lock(mutex_);
    void* din = staging(0, mat_bytes(input));
    void* dout = staging(1, mat_bytes(top_blobs[0]));
    if (!din || !dout)
        return -100;
    cudaError_t err = upload(din, input);
    int rc = AWA_OK;
    if (err == cudaSuccess)
        rc = awa_window_attention(plan_, bf16 ? AWA_PREC_BF16 : AWA_PREC_FP32, heads, input.w,
                                  dtype_of(input.elemsize), din, (int64_t)input.cstep, dtype_of(out_elem), dout,
                                  (int64_t)top_blobs[0].cstep, nullptr);
    if (err == cudaSuccess && rc == AWA_OK)
        err = download(top_blobs[0], dout);
    return finish(err, rc, "SeedVR2WindowAttention");
}

int SeedVR2WindowAttention::forward_cuda(const std::vector<CudaBlob>& bottom_blobs, std::vector<CudaBlob>& top_blobs,
                                         const CudaOption& opt) const
{
    if (bottom_blobs.size() != 1 || !plan_)
        return -1;
    const CudaBlob& input = bottom_blobs[0];
    if (input.dims != 3 || (input.elemsize != 4u && input.elemsize != 2u) || input.w <= 0 || input.h <= 0 ||
        input.h % 3 != 0 || input.c != info_.sequence_tokens)
        return -1;
    const size_t out_elem = opt.use_bf16_storage ? 2u : 4u;
    const int heads = input.h / 3;
    top_blobs.resize(1);
    if (seedvr2::cuda_blob_create(top_blobs[0], 3, input.w, heads, 1, info_.sequence_tokens, out_elem))
        return -100;
    return to_ncnn_status(awa_window_attention(plan_, opt.use_bf16_storage ? AWA_PREC_BF16 : AWA_PREC_FP32, heads,
                                               input.w, dtype_of(input.elemsize), input.data, (int64_t)input.cstep,
                                               dtype_of(out_elem), top_blobs[0].data, (int64_t)top_blobs[0].cstep,
                                               opt.stream),
                          "SeedVR2WindowAttention");
}

// ------------------------------------------------------------------ Unpack
SeedVR2AWAUnpack::SeedVR2AWAUnpack() {}

SeedVR2AWAUnpack::SeedVR2AWAUnpack(const seedvr2::AwaRuntimeSpec& runtime_spec) : seedvr2::AwaLayerBase(runtime_spec) {}

int SeedVR2AWAUnpack::load_param(const ncnn::ParamDict& pd)
{
    return load_common_params(pd, 126);
}

namespace
{

// The video output of Unpack. Without NCNN_BATCH it is (w=d, h=H, c=N_v):
// one token per channel, cstep apart. With NCNN_BATCH it is the 4-D batched
// blob (w=d, h=H, d=W, c=H_grid, n=T) of awa_layers.cpp:655-656, token
// (t, y, x) at t*nstep + y*cstep + x*H*d: tokens are evenly strided inside a
// frame when cstep is W*H*d, and frames are nstep apart, which the 4 KiB batch
// alignment can make more than a frame's size. awa_unpack writes one token
// stride, so frames that are not evenly strided go through a dense staging
// buffer and a pitched copy per frame.
struct VideoTarget
{
    int64_t token_stride = 0;  // stride for awa_unpack when writing in place
    bool in_place = true;      // else: dense staging, then copy_frames()
};

template <typename Blob>
VideoTarget video_target(const Blob& out, int heads, int head_dim, const awa_plan_info& info)
{
    VideoTarget t;
    const int64_t row = (int64_t)heads * head_dim;
#if NCNN_BATCH
    const bool rows_even = out.cstep == (size_t)row * info.source_w;
    const bool frames_even = out.nstep == out.cstep * (size_t)info.source_h;
    t.in_place = rows_even && (frames_even || info.source_t == 1);
    t.token_stride = row;
#else
    (void)row;
    (void)info;
    t.token_stride = (int64_t)out.cstep;
#endif
    return t;
}

// Dense [N_v][H*d] rows at src -> the batched video blob at dst, one pitched
// copy per frame (rows of one grid line are contiguous in both).
template <typename Blob>
cudaError_t copy_frames(void* dst, const Blob& out, const void* src, int heads, int head_dim,
                        const awa_plan_info& info, cudaMemcpyKind kind, cudaStream_t stream)
{
    const size_t es = out.elemsize;
    const size_t line = (size_t)heads * head_dim * info.source_w * es;
    for (int t = 0; t < info.source_t; t++)
    {
        const unsigned char* s = static_cast<const unsigned char*>(src) + (size_t)t * info.source_h * line;
        unsigned char* d = static_cast<unsigned char*>(dst) + (size_t)t * out.nstep * es;
        const cudaError_t err = cudaMemcpy2DAsync(d, out.cstep * es, s, line, line, info.source_h, kind, stream);
        if (err != cudaSuccess)
            return err;
    }
    return cudaSuccess;
}

}  // namespace

int SeedVR2AWAUnpack::forward(const std::vector<ncnn::Mat>& bottom_blobs, std::vector<ncnn::Mat>& top_blobs,
                              const ncnn::Option& opt) const
{
    if (bottom_blobs.size() != 1 || !plan_)
        return -1;
    const ncnn::Mat& packed = bottom_blobs[0];
    if (packed.dims != 3 || packed.elempack != 1 || (packed.elemsize != 4u && packed.elemsize != 2u) ||
        packed.w <= 0 || packed.h <= 0 || packed.c != info_.sequence_tokens)
        return -1;
    const int heads = packed.h;
    const int head_dim = packed.w;
    const size_t out_elem = bf16_blocks(opt) ? 2u : 4u;  // bf16 blocks cast both outputs (awa_layers.cpp:832-837)
    top_blobs.resize(2);
#if NCNN_BATCH
    top_blobs[0].create(head_dim, heads, info_.source_w, info_.source_h, out_elem, 1, info_.source_t,
                        opt.blob_allocator);
#else
    top_blobs[0].create(head_dim, heads, info_.source_tokens, out_elem, opt.blob_allocator);
#endif
    top_blobs[1].create(head_dim, heads, info_.text_tokens, out_elem, opt.blob_allocator);
    if (top_blobs[0].empty() || top_blobs[1].empty())
        return -100;
    const VideoTarget target = video_target(top_blobs[0], heads, head_dim, info_);
    std::lock_guard<std::mutex> lock(mutex_);
    void* din = staging(0, mat_bytes(packed));
    void* dv = staging(1, target.in_place ? mat_bytes(top_blobs[0])
                                          : (size_t)info_.source_tokens * heads * head_dim * out_elem);
    void* dt = staging(2, mat_bytes(top_blobs[1]));
    if (!din || !dv || !dt)
        return -100;
    cudaError_t err = upload(din, packed);
    int rc = AWA_OK;
    if (err == cudaSuccess)
        rc = awa_unpack(plan_, heads, head_dim, dtype_of(packed.elemsize), din, (int64_t)packed.cstep,
                        dtype_of(out_elem), dv, target.token_stride, dt, (int64_t)top_blobs[1].cstep, nullptr);
    if (err == cudaSuccess && rc == AWA_OK)
        err = target.in_place ? download(top_blobs[0], dv)
                              : copy_frames(top_blobs[0].data, top_blobs[0], dv, heads, head_dim, info_,
                                            cudaMemcpyDeviceToHost, nullptr);
    if (err == cudaSuccess && rc == AWA_OK)
        err = download(top_blobs[1], dt);
    return finish(err, rc, "SeedVR2AWAUnpack");
}

int SeedVR2AWAUnpack::forward_cuda(const std::vector<CudaBlob>& bottom_blobs, std::vector<CudaBlob>& top_blobs,
                                   const CudaOption& opt) const
{
    if (bottom_blobs.size() != 1 || !plan_)
        return -1;
    const CudaBlob& packed = bottom_blobs[0];
    if (packed.dims != 3 || (packed.elemsize != 4u && packed.elemsize != 2u) || packed.w <= 0 || packed.h <= 0 ||
        packed.c != info_.sequence_tokens)
        return -1;
    const int heads = packed.h;
    const int head_dim = packed.w;
    const size_t out_elem = opt.use_bf16_storage ? 2u : 4u;
    top_blobs.resize(2);
#if NCNN_BATCH
    const int video_rc = seedvr2::cuda_blob_create(top_blobs[0], 4, head_dim, heads, info_.source_w,
                                                   info_.source_h, out_elem, info_.source_t);
#else
    const int video_rc = seedvr2::cuda_blob_create(top_blobs[0], 3, head_dim, heads, 1, info_.source_tokens, out_elem);
#endif
    if (video_rc || seedvr2::cuda_blob_create(top_blobs[1], 3, head_dim, heads, 1, info_.text_tokens, out_elem))
        return -100;
    const VideoTarget target = video_target(top_blobs[0], heads, head_dim, info_);
    void* dv = top_blobs[0].data;
    if (!target.in_place)
    {
        std::lock_guard<std::mutex> lock(mutex_);
        dv = staging(5, (size_t)info_.source_tokens * heads * head_dim * out_elem);
        if (!dv)
            return -100;
    }
    int rc = awa_unpack(plan_, heads, head_dim, dtype_of(packed.elemsize), packed.data, (int64_t)packed.cstep,
                        dtype_of(out_elem), dv, target.token_stride, top_blobs[1].data, (int64_t)top_blobs[1].cstep,
                        opt.stream);
    if (rc == AWA_OK && !target.in_place &&
        copy_frames(top_blobs[0].data, top_blobs[0], dv, heads, head_dim, info_, cudaMemcpyDeviceToDevice,
                    static_cast<cudaStream_t>(opt.stream)) != cudaSuccess)
    {
        std::fprintf(stderr, "SeedVR2AWAUnpack: batched video copy failed\n");
        return -1;
    }
    return to_ncnn_status(rc, "SeedVR2AWAUnpack");
}

// ------------------------------------------------------------------ registration
DEFINE_LAYER_CREATOR(SeedVR2AWAPack)
DEFINE_LAYER_CREATOR(SeedVR2AWAUnpack)
DEFINE_LAYER_CREATOR(SeedVR2MMRoPE)
DEFINE_LAYER_CREATOR(SeedVR2WindowAttention)

namespace
{

template <typename L>
ncnn::Layer* runtime_creator(void* userdata)
{
    return new L(*static_cast<const seedvr2::AwaRuntimeSpec*>(userdata));
}

}  // namespace

void register_seedvr2_awa_layers(ncnn::Net& net)
{
    net.register_custom_layer("SeedVR2AWAPack", SeedVR2AWAPack_layer_creator);
    net.register_custom_layer("SeedVR2AWAUnpack", SeedVR2AWAUnpack_layer_creator);
    net.register_custom_layer("SeedVR2MMRoPE", SeedVR2MMRoPE_layer_creator);
    net.register_custom_layer("SeedVR2WindowAttention", SeedVR2WindowAttention_layer_creator);
}

void register_seedvr2_awa_layers(ncnn::Net& net, const seedvr2::AwaRuntimeSpec* runtime_spec)
{
    if (!runtime_spec)
    {
        register_seedvr2_awa_layers(net);
        return;
    }
    void* userdata = const_cast<seedvr2::AwaRuntimeSpec*>(runtime_spec);
    net.register_custom_layer("SeedVR2AWAPack", runtime_creator<SeedVR2AWAPack>, nullptr, userdata);
    net.register_custom_layer("SeedVR2AWAUnpack", runtime_creator<SeedVR2AWAUnpack>, nullptr, userdata);
    net.register_custom_layer("SeedVR2MMRoPE", runtime_creator<SeedVR2MMRoPE>, nullptr, userdata);
    net.register_custom_layer("SeedVR2WindowAttention", runtime_creator<SeedVR2WindowAttention>, nullptr, userdata);
}
