// chain_driver.cpp -- C entry point that drives the four ncnn layer classes
// the way a DiT block graph does (dit_stack.cpp:180 registration,
// export_dit_block.py:578-644 layer lines): register_seedvr2_awa_layers(),
// create through the Net, load_param with ParamDict ids 0-8, then
// Pack -> MMRoPE -> WindowAttention -> Unpack on ncnn Mats (host blobs) or on
// CudaBlobs (device blobs). Used by the integration tests and by callers that
// want the whole chain behind one call.
#include <cstring>
#include <vector>

#include <cuda_runtime.h>

#include "awa_layers.h"
#include "net.h"

namespace
{

// Dense [tokens][3][H][d] host array -> QKV blob in encoding `layout`
// (0: w=d,h=3H,c=N; 1: w=d,h=H,c=3N; 2: dims 4, w=d,h=H,d=3,c=N).
void fill_qkv(ncnn::Mat& m, const void* src, int tokens, int heads, int head_dim, int layout, size_t elemsize)
{
    const size_t row = (size_t)heads * head_dim * elemsize;
    const unsigned char* s = static_cast<const unsigned char*>(src);
    if (layout == 0)
    {
        m.create(head_dim, 3 * heads, tokens, elemsize);
        for (int t = 0; t < tokens; t++)
            std::memcpy(m.channel(t).data, s + (size_t)t * 3 * row, 3 * row);
    }
    else if (layout == 1)
    {
        m.create(head_dim, heads, 3 * tokens, elemsize);
        for (int q = 0; q < 3; q++)
            for (int t = 0; t < tokens; t++)
                std::memcpy(m.channel(q * tokens + t).data, s + ((size_t)t * 3 + q) * row, row);
    }
    else
    {
        m.create(head_dim, heads, 3, tokens, elemsize);
        for (int t = 0; t < tokens; t++)
            std::memcpy(m.channel(t).data, s + (size_t)t * 3 * row, 3 * row);
    }
}

void read_dense(const ncnn::Mat& m, void* dst)
{
    const size_t plane = (size_t)m.w * m.h * m.elemsize;
    for (int c = 0; c < m.c; c++)
        std::memcpy(static_cast<unsigned char*>(dst) + (size_t)c * plane, m.channel(c).data, plane);
}

ncnn::Mat to_mat(const seedvr2::CudaBlob& b)
{
    ncnn::Mat m;
    if (b.dims == 1)
        m.create(b.w, b.elemsize);
    else
        m.create(b.w, b.h, b.c, b.elemsize);
    cudaMemcpy(m.data, b.data, m.dims == 1 ? (size_t)b.w * b.elemsize : b.cstep * b.c * b.elemsize,
               cudaMemcpyDeviceToHost);
    return m;
}

seedvr2::CudaBlob to_blob(const ncnn::Mat& m)
{
    seedvr2::CudaBlob b;
    seedvr2::cuda_blob_create(b, m.dims, m.w, m.h, m.d, m.c, m.elemsize);
    if (b.data)
        cudaMemcpy(b.data, m.data, m.dims >= 3 ? m.cstep * m.c * m.elemsize : (size_t)m.w * m.h * m.elemsize,
                   cudaMemcpyHostToDevice);
    b.cstep = m.cstep;
    return b;
}

}  // namespace

extern "C" {

// params: ParamDict ids 0-8. Inputs are dense host arrays of elemsize bytes per
// element (4 = fp32, 2 = bf16). device_blobs != 0 runs forward_cuda on device
// copies. Outputs (dense, output element size = 2 when bf16 else 4) may be NULL.
// Returns the first non-zero layer status.
int awa_ncnn_run_chain(const int* params, int heads, int head_dim, int layout, int use_runtime_spec, int bf16,
                       int device_blobs, int input_elemsize, const void* video_qkv, const void* text_qkv,
                       void* packed, float* cu_seqlens, void* roped, void* attended, void* video_out, void* text_out)
{
    ncnn::Net net;
    seedvr2::AwaRuntimeSpec spec;
    spec.source_t = params[0];
    spec.source_h = params[1];
    spec.source_w = params[2];
    spec.video_tokens = params[0] * params[1] * params[2];
    register_seedvr2_awa_layers(net, use_runtime_spec ? &spec : nullptr);
    const char* types[4] = {"SeedVR2AWAPack", "SeedVR2MMRoPE", "SeedVR2WindowAttention", "SeedVR2AWAUnpack"};
    ncnn::Layer* layers[4];
    ncnn::ParamDict pd;
    for (int id = 0; id < 9; id++)
        pd.set(id, params[id]);
    if (use_runtime_spec)
    {
        pd.set(0, -1);
        pd.set(1, -1);
        pd.set(2, -1);
    }
    int rc = 0;
    for (int i = 0; i < 4; i++)
    {
        layers[i] = net.create_custom_layer(types[i]);
        if (rc == 0)
            rc = layers[i]->load_param(pd);
    }
    const int video_tokens = params[0] * params[1] * params[2];
    if (rc == 0)
    {
        ncnn::Option opt;
        opt.use_bf16_storage = bf16 != 0;
        std::vector<ncnn::Mat> in(2), t0, t1, t2, t3;
        fill_qkv(in[0], video_qkv, video_tokens, heads, head_dim, layout, (size_t)input_elemsize);
        fill_qkv(in[1], text_qkv, params[6], heads, head_dim, layout, (size_t)input_elemsize);
        if (!device_blobs)
        {
            rc = layers[0]->forward(in, t0, opt);
            std::vector<ncnn::Mat> r_in(1, rc == 0 ? t0[0] : ncnn::Mat());
            if (rc == 0)
                rc = layers[1]->forward(r_in, t1, opt);
            if (rc == 0)
                rc = layers[2]->forward(t1, t2, opt);
            if (rc == 0)
                rc = layers[3]->forward(t2, t3, opt);
        }
        else
        {
            seedvr2::CudaOption copt;
            copt.use_bf16_storage = bf16 != 0;
            std::vector<seedvr2::CudaBlob> b_in(2), b0, b1, b2, b3;
            b_in[0] = to_blob(in[0]);
            b_in[1] = to_blob(in[1]);
            rc = static_cast<SeedVR2AWAPack*>(layers[0])->forward_cuda(b_in, b0, copt);
            std::vector<seedvr2::CudaBlob> r_in(1);
            if (rc == 0)
            {
                r_in[0] = b0[0];
                r_in[0].owned = false;
                rc = static_cast<SeedVR2MMRoPE*>(layers[1])->forward_cuda(r_in, b1, copt);
            }
            if (rc == 0)
                rc = static_cast<SeedVR2WindowAttention*>(layers[2])->forward_cuda(b1, b2, copt);
            if (rc == 0)
                rc = static_cast<SeedVR2AWAUnpack*>(layers[3])->forward_cuda(b2, b3, copt);
            if (rc == 0 && cudaDeviceSynchronize() != cudaSuccess)
                rc = -1;
            if (rc == 0)
            {
                t0.push_back(to_mat(b0[0]));
                t0.push_back(to_mat(b0[1]));
                t1.push_back(to_mat(b1[0]));
                t2.push_back(to_mat(b2[0]));
                t3.push_back(to_mat(b3[0]));
                t3.push_back(to_mat(b3[1]));
            }
            for (auto* v : {&b_in, &b0, &b1, &b2, &b3})
                for (auto& b : *v)
                    seedvr2::cuda_blob_free(b);
        }
        if (rc == 0)
        {
            if (packed)
                read_dense(t0[0], packed);
            if (cu_seqlens)
                std::memcpy(cu_seqlens, t0[1].data, sizeof(float) * t0[1].w);
            if (roped)
                read_dense(t1[0], roped);
            if (attended)
                read_dense(t2[0], attended);
            if (video_out)
                read_dense(t3[0], video_out);
            if (text_out)
                read_dense(t3[1], text_out);
        }
    }
    for (int i = 0; i < 4; i++)
        net.destroy_custom_layer(types[i], layers[i]);
    return rc;
}

}  // extern "C"
