// awa_layers.h -- ncnn custom layers of SeedVR2's adaptive window attention,
// backed by the B200 CUDA library (include/awa_b200.h).
//
// Same type names, constructors, ParamDict ids 0-8, blob arity and shapes,
// runtime-spec creator userdata and return codes as the reference layers
// (HGinkgo/SeedVR2-ncnn src/awa/awa_layers.h:17-223), so an ncnn graph that
// registers these instead of the reference's runs unchanged:
//
//   SeedVR2AWAPack          2 -> 2   (video QKV, text QKV) -> (packed QKV, cu_seqlens)
//   SeedVR2MMRoPE           1 -> 1
//   SeedVR2WindowAttention  1 -> 1
//   SeedVR2AWAUnpack        1 -> 2   attended -> (video, text)
//
// forward(Mat) takes host blobs (as the reference's CPU forward does) and runs
// the CUDA kernels in between host<->device copies. forward_cuda(CudaBlob)
// is the device path (the CUDA counterpart of the reference's VkMat forward):
// blobs stay in HBM and all work is enqueued on the given stream.
// Precision follows the ncnn option of the block, as in the reference
// (awa_layers.cpp:184-187): use_bf16_storage / use_bf16_packed select bf16
// blobs and tensor-core attention, otherwise everything is fp32.
#pragma once

#include <mutex>
#include <vector>

#include "awa_b200.h"
#include "layer.h"

namespace ncnn
{
class Net;
}

namespace seedvr2
{

struct AwaWindow final
{
    int t0 = 0;
    int t1 = 0;
    int h0 = 0;
    int h1 = 0;
    int w0 = 0;
    int w1 = 0;
};

// Resolution metadata owned by one loaded ncnn::Net session (awa_layers.h:31-39).
struct AwaRuntimeSpec final
{
    int source_t = 0;
    int source_h = 0;
    int source_w = 0;
    int video_tokens = 0;

    bool valid() const;
};

// Windows in the order the layers use (make_awa_windows, awa_layers.cpp:347-359).
std::vector<AwaWindow> make_awa_windows(int source_t, int source_h, int source_w, int windows_t, int windows_h,
                                        int windows_w, bool shifted);

// A device blob: ncnn Mat geometry over memory on the current CUDA device.
struct CudaBlob
{
    void* data = nullptr;
    int dims = 0;
    int w = 0;
    int h = 0;
    int d = 1;
    int c = 0;
    size_t elemsize = 4;
    size_t cstep = 0;
    int n = 1;         // batch items (NCNN_BATCH layouts)
    size_t nstep = 0;  // elements between batch items
    bool owned = false;  // allocated by a layer (release with cuda_blob_free)
};

// Layout-compatible with ncnn::Mat::create: cstep aligned to 16 bytes for
// dims >= 3; with n > 1 (the batched form) nstep is cstep * c rounded up to
// 4 KiB, as the Mat subset in ncnn_compat/ncnn does.
int cuda_blob_create(CudaBlob& blob, int dims, int w, int h, int d, int c, size_t elemsize, int n = 1);
void cuda_blob_free(CudaBlob& blob);

struct CudaOption
{
    awa_stream_t stream = nullptr;
    bool use_bf16_storage = false;
};

// Shared state and helpers of the four layers.
class AwaLayerBase : public ncnn::Layer
{
public:
    AwaLayerBase();
    explicit AwaLayerBase(const AwaRuntimeSpec& runtime_spec);
    ~AwaLayerBase() override;

protected:
    int load_common_params(const ncnn::ParamDict& pd, int rope_dim);
    const awa_plan* plan() const { return plan_; }
    // Device staging for the host-blob forward (grow-only, per layer).
    void* staging(int slot, size_t bytes) const;

    bool has_runtime_spec_ = false;
    AwaRuntimeSpec runtime_spec_;
    awa_plan* plan_ = nullptr;
    awa_plan_info info_{};
    mutable std::mutex mutex_;
    mutable void* staging_[6] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
    mutable size_t staging_bytes_[6] = {0, 0, 0, 0, 0, 0};
};

} // namespace seedvr2

class SeedVR2AWAPack final : public seedvr2::AwaLayerBase
{
public:
    SeedVR2AWAPack();
    explicit SeedVR2AWAPack(const seedvr2::AwaRuntimeSpec& runtime_spec);

    int load_param(const ncnn::ParamDict& pd) override;
    int forward(const std::vector<ncnn::Mat>& bottom_blobs, std::vector<ncnn::Mat>& top_blobs,
                const ncnn::Option& opt) const override;
    int forward_cuda(const std::vector<seedvr2::CudaBlob>& bottom_blobs, std::vector<seedvr2::CudaBlob>& top_blobs,
                     const seedvr2::CudaOption& opt) const;
};

class SeedVR2AWAUnpack final : public seedvr2::AwaLayerBase
{
public:
    SeedVR2AWAUnpack();
    explicit SeedVR2AWAUnpack(const seedvr2::AwaRuntimeSpec& runtime_spec);

    int load_param(const ncnn::ParamDict& pd) override;
    int forward(const std::vector<ncnn::Mat>& bottom_blobs, std::vector<ncnn::Mat>& top_blobs,
                const ncnn::Option& opt) const override;
    int forward_cuda(const std::vector<seedvr2::CudaBlob>& bottom_blobs, std::vector<seedvr2::CudaBlob>& top_blobs,
                     const seedvr2::CudaOption& opt) const;
};

class SeedVR2MMRoPE final : public seedvr2::AwaLayerBase
{
public:
    SeedVR2MMRoPE();
    explicit SeedVR2MMRoPE(const seedvr2::AwaRuntimeSpec& runtime_spec);

    int load_param(const ncnn::ParamDict& pd) override;
    int forward(const std::vector<ncnn::Mat>& bottom_blobs, std::vector<ncnn::Mat>& top_blobs,
                const ncnn::Option& opt) const override;
    int forward_cuda(const std::vector<seedvr2::CudaBlob>& bottom_blobs, std::vector<seedvr2::CudaBlob>& top_blobs,
                     const seedvr2::CudaOption& opt) const;

private:
    int rope_dim_ = 0;
};

class SeedVR2WindowAttention final : public seedvr2::AwaLayerBase
{
public:
    SeedVR2WindowAttention();
    explicit SeedVR2WindowAttention(const seedvr2::AwaRuntimeSpec& runtime_spec);

    int load_param(const ncnn::ParamDict& pd) override;
    int forward(const std::vector<ncnn::Mat>& bottom_blobs, std::vector<ncnn::Mat>& top_blobs,
                const ncnn::Option& opt) const override;
    int forward_cuda(const std::vector<seedvr2::CudaBlob>& bottom_blobs, std::vector<seedvr2::CudaBlob>& top_blobs,
                     const seedvr2::CudaOption& opt) const;
};

void register_seedvr2_awa_layers(ncnn::Net& net);
void register_seedvr2_awa_layers(ncnn::Net& net, const seedvr2::AwaRuntimeSpec* runtime_spec);
