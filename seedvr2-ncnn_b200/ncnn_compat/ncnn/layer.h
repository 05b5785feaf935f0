// Subset of Tencent/ncnn's layer.h (Layer base class, creator typedefs,
// DEFINE_LAYER_CREATOR) that the SeedVR2 AWA layer classes use; see mat.h.
#pragma once

#include <vector>

#include "mat.h"
#include "option.h"
#include "paramdict.h"

namespace ncnn
{

class VulkanDevice;

class Layer
{
public:
    Layer() {}
    virtual ~Layer() {}

    virtual int load_param(const ParamDict&) { return 0; }
    virtual int forward(const std::vector<Mat>&, std::vector<Mat>&, const Option&) const { return -1; }

    bool one_blob_only = false;
    bool support_inplace = false;
    bool support_vulkan = false;
    bool support_packing = false;
    bool support_bf16_storage = false;
    bool support_fp16_storage = false;
    bool support_int8_storage = false;
    bool support_image_storage = false;
    bool support_tensor_storage = false;
    bool support_any_packing = false;
    bool support_vulkan_packing = false;
    bool support_vulkan_any_packing = false;
    bool support_batch = false;
    void* userdata = 0;
    int typeindex = -1;
    const VulkanDevice* vkdev = 0;
};

typedef Layer* (*layer_creator_func)(void*);
typedef void (*layer_destroyer_func)(Layer*, void*);

} // namespace ncnn

#define DEFINE_LAYER_CREATOR(name)                          \
    ::ncnn::Layer* name##_layer_creator(void* /*userdata*/) \
    {                                                       \
        return new name;                                    \
    }
