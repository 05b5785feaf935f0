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
// (0: w=d,h=3H,c=N; 1: w=d,h=H,c=3N; 2: dims 4, w=d,h=H,d=3,c=N; 3, NCNN_BATCH
// builds only: w=d,h=H,c=3,n=N, one token per batch item).
bool fill_qkv(ncnn::Mat& m, const void* src, int tokens, int heads, int head_dim, int layout, size_t elemsize)
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
    else if (layout == 2)
    {
        m.create(head_dim, heads, 3, tokens, elemsize);
        for (int t = 0; t < tokens; t++)
            std::memcpy(m.channel(t).data, s + (size_t)t * 3 * row, 3 * row);
    }
#if NCNN_BATCH
    else if (layout == 3)
    {
        m.create(head_dim, heads, 3, elemsize, 1, tokens);
        for (int t = 0; t < tokens; t++)
            for (int q = 0; q < 3; q++)
                std::memcpy(m.batch(t).channel(q).data, s + ((size_t)t * 3 + q) * row, row);
    }
#endif
    else
        return false;
    return true;
}

// Any blob with Mat geometry -> dense host rows. dims 3: [c][h][w];
// dims 4 (with batch items n): [n][c][d][h][w].
void read_dense(const ncnn::Mat& m, void* dst)
{
    unsigned char* out = static_cast<unsigned char*>(dst);
    if (m.dims < 3)
    {
        std::memcpy(out, m.data, (size_t)m.w * m.h * m.elemsize);
        return;
    }
    const size_t plane = (size_t)m.w * m.h * m.elemsize;
    const int depth = m.dims == 4 ? m.d : 1;
    for (int b = 0; b < m.n; b++)
        for (int c = 0; c < m.c; c++)
        {
            const unsigned char* src = static_cast<const unsigned char*>(m.data) + (b * m.nstep + c * m.cstep) * m.elemsize;
            std::memcpy(out, src, plane * depth);
            out += plane * depth;
        }
}

size_t storage_bytes(int dims, int w, int h, int c, int n, size_t cstep, size_t nstep, size_t elemsize)
{
    const size_t one = dims >= 3 ? cstep * c : (size_t)w * h;
    return (n > 1 ? nstep * (size_t)(n - 1) + one : one) * elemsize;
}

// Device blob -> host Mat of the same geometry (cstep / nstep kept).
ncnn::Mat to_mat(const seedvr2::CudaBlob& b)
{
    ncnn::Mat m;
    if (b.dims == 1)
        m.create(b.w, b.elemsize);
    else if (b.dims == 4 && b.n > 1)
        m.create(b.w, b.h, b.d, b.c, b.elemsize, 1, b.n);
    else if (b.dims == 4)
        m.create(b.w, b.h, b.d, b.c, b.elemsize);
    else
        m.create(b.w, b.h, b.c, b.elemsize);
    if (m.cstep != b.cstep || (b.n > 1 && m.nstep != b.nstep))
        return ncnn::Mat();
    cudaMemcpy(m.data, b.data, storage_bytes(b.dims, b.w, b.h, b.c, b.n, b.cstep, b.nstep, b.elemsize),
               cudaMemcpyDeviceToHost);
    return m;
}

// Host Mat -> device blob of the same geometry.
seedvr2::CudaBlob to_blob(const ncnn::Mat& m)
{
    seedvr2::CudaBlob b;
    seedvr2::cuda_blob_create(b, m.dims, m.w, m.h, m.d, m.c, m.elemsize, m.n);
    if (b.data)
        cudaMemcpy(b.data, m.data, storage_bytes(m.dims, m.w, m.h, m.c, m.n, m.cstep, m.nstep, m.elemsize),
                   cudaMemcpyHostToDevice);
    b.cstep = m.cstep;
    b.nstep = m.nstep;
    return b;
}

}  // namespace

extern "C" {

// 1 when this library was built with NCNN_BATCH (batched QKV and video blobs).
int awa_ncnn_batch_build(void)
{
#if NCNN_BATCH
    return 1;
#else
    return 0;
#endif
}

// params: ParamDict ids 0-8. Inputs are dense host arrays of elemsize bytes per
// element (4 = fp32, 2 = bf16), written into the QKV blob encoding `layout`
// (see fill_qkv; 3 needs a library built with NCNN_BATCH). device_blobs != 0
// runs forward_cuda on device copies. Outputs (dense, output element size = 2
// when bf16 else 4) may be NULL. Returns the first non-zero layer status, -1
// for a layout this build does not have.
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
        if (!fill_qkv(in[0], video_qkv, video_tokens, heads, head_dim, layout, (size_t)input_elemsize) ||
            !fill_qkv(in[1], text_qkv, params[6], heads, head_dim, layout, (size_t)input_elemsize))
            rc = -1;
        else if (!device_blobs)
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
