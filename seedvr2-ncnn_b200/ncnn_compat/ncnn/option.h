// Subset of Tencent/ncnn's Option used by the SeedVR2 AWA layer classes.
#pragma once

namespace ncnn
{

class Allocator;
class VkAllocator;

class Option
{
public:
    int num_threads = 1;
    Allocator* blob_allocator = 0;
    Allocator* workspace_allocator = 0;
    bool use_vulkan_compute = false;
    bool use_bf16_storage = false;
    bool use_bf16_packed = false;
    bool use_fp16_storage = false;
    bool use_fp16_packed = false;
    bool use_fp16_arithmetic = false;
    bool use_packing_layout = false;
};

} // namespace ncnn
