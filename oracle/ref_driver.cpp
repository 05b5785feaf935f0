// ref_driver.cpp -- C entry points around the reference's OWN CPU forward
// (src/awa/awa_layers.cpp of HGinkgo/SeedVR2-ncnn, compiled unmodified with
// NCNN_VULKAN=0 against the library's ncnn API subset in
// seedvr2-ncnn_b200/ncnn_compat/ncnn). TEST INFRASTRUCTURE: used by tests/ to
// pin the C restatement (awa_oracle.c) and by bench.py's reference arm.
//
// The chain is driven the way an ncnn graph drives it (dit_stack.cpp:180,
// export_dit_block.py:578-644): layers are created through
// register_seedvr2_awa_layers() + Net, configured with load_param(ParamDict
// ids 0-8), and run with forward(bottoms, tops, opt). Dense fp32 arrays are
// copied into / out of ncnn Mats (whose cstep may be padded).
#include <chrono>
#include <cstdio>
#include <cstring>
#include <vector>

#include "awa_layers.h"
#include "net.h"

namespace
{

struct RefChain
{
    ncnn::Net net;
    ncnn::Layer* pack = 0;
    ncnn::Layer* rope = 0;
    ncnn::Layer* attention = 0;
    ncnn::Layer* unpack = 0;
    int source_tokens = 0;
    int text_tokens = 0;
    int heads = 0;
    int head_dim = 0;
    int layout = 0;
    double seconds[4] = {0, 0, 0, 0};

    ~RefChain()
    {
        net.destroy_custom_layer("SeedVR2AWAPack", pack);
        net.destroy_custom_layer("SeedVR2MMRoPE", rope);
        net.destroy_custom_layer("SeedVR2WindowAttention", attention);
        net.destroy_custom_layer("SeedVR2AWAUnpack", unpack);
    }
};

// Copy a dense [tokens][3][H][d] array into one of the QKV blob encodings
// accepted by describe_qkv_layout (awa_layers.cpp:124-170):
//   layout 0: dims 3, w=d, h=3H, c=tokens
//   layout 1: dims 3, w=d, h=H,  c=3*tokens (all q rows, then k, then v)
//   layout 2: dims 4, w=d, h=H,  d=3, c=tokens
//   layout 3: dims 3, w=d, h=H,  c=3, n=tokens (NCNN_BATCH builds only)
// Returns false for a layout this build does not have.
bool fill_qkv(ncnn::Mat& m, const float* src, int tokens, int heads, int head_dim, int layout)
{
    const size_t head_row = (size_t)heads * head_dim;
    if (layout == 0)
    {
        m.create(head_dim, 3 * heads, tokens, 4u);
        for (int t = 0; t < tokens; t++)
            std::memcpy(m.channel(t).data, src + (size_t)t * 3 * head_row, 3 * head_row * sizeof(float));
    }
    else if (layout == 1)
    {
        m.create(head_dim, heads, 3 * tokens, 4u);
        for (int qkv = 0; qkv < 3; qkv++)
            for (int t = 0; t < tokens; t++)
                std::memcpy(m.channel(qkv * tokens + t).data, src + ((size_t)t * 3 + qkv) * head_row,
                            head_row * sizeof(float));
    }
    else if (layout == 2)
    {
        m.create(head_dim, heads, 3, tokens, 4u);
        for (int t = 0; t < tokens; t++)
            std::memcpy(m.channel(t).data, src + (size_t)t * 3 * head_row, 3 * head_row * sizeof(float));
    }
#if NCNN_BATCH
    else if (layout == 3)
    {
        m.create(head_dim, heads, 3, 4u, 1, tokens);
        for (int t = 0; t < tokens; t++)
            for (int qkv = 0; qkv < 3; qkv++)
                std::memcpy(m.batch(t).channel(qkv).data, src + ((size_t)t * 3 + qkv) * head_row,
                            head_row * sizeof(float));
    }
#endif
    else
        return false;
    return true;
}

// Copy a Mat to dense rows: dims 3 (w, h, c) -> [c][h][w]; dims 4 with batch
// items (the NCNN_BATCH video output, w, h, d, c, n) -> [n][c][d][h][w].
void read_dense(const ncnn::Mat& m, float* dst)
{
    const size_t plane = (size_t)m.w * m.h * (m.dims == 4 ? m.d : 1);
    for (int b = 0; b < m.n; b++)
        for (int c = 0; c < m.c; c++)
        {
            const float* src = static_cast<const float*>(m.data) + b * m.nstep + c * m.cstep;
            std::memcpy(dst, src, plane * sizeof(float));
            dst += plane;
        }
}

double now_seconds()
{
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

} // namespace

extern "C" {

// 1 when the reference was compiled with NCNN_BATCH.
int ref_batch_build(void)
{
#if NCNN_BATCH
    return 1;
#else
    return 0;
#endif
}

int ref_make_windows(int source_t, int source_h, int source_w, int num_t, int num_h, int num_w, int shifted,
                     int* out6, int capacity)
{
    const std::vector<seedvr2::AwaWindow> windows =
        seedvr2::make_awa_windows(source_t, source_h, source_w, num_t, num_h, num_w, shifted != 0);
    for (size_t i = 0; i < windows.size() && (int)i < capacity; i++)
    {
        int* o = out6 + 6 * i;
        o[0] = windows[i].t0;
        o[1] = windows[i].t1;
        o[2] = windows[i].h0;
        o[3] = windows[i].h1;
        o[4] = windows[i].w0;
        o[5] = windows[i].w1;
    }
    return (int)windows.size();
}

// params: T,H,W, nt,nh,nw, text_tokens, shifted, rope_dim (ParamDict ids 0-8).
// use_runtime_spec != 0 writes ids 0-2 as -1 and passes an AwaRuntimeSpec
// through register_seedvr2_awa_layers (the dynamic-package path).
void* ref_chain_create(const int* params, int heads, int head_dim, int layout, int use_runtime_spec, int* status)
{
    RefChain* chain = new RefChain();
    static thread_local seedvr2::AwaRuntimeSpec spec;
    spec.source_t = params[0];
    spec.source_h = params[1];
    spec.source_w = params[2];
    spec.video_tokens = params[0] * params[1] * params[2];
    register_seedvr2_awa_layers(chain->net, use_runtime_spec ? &spec : nullptr);
    chain->pack = chain->net.create_custom_layer("SeedVR2AWAPack");
    chain->rope = chain->net.create_custom_layer("SeedVR2MMRoPE");
    chain->attention = chain->net.create_custom_layer("SeedVR2WindowAttention");
    chain->unpack = chain->net.create_custom_layer("SeedVR2AWAUnpack");
    ncnn::ParamDict pd;
    for (int id = 0; id < 8; id++)
        pd.set(id, params[id]);
    if (use_runtime_spec)
    {
        pd.set(0, -1);
        pd.set(1, -1);
        pd.set(2, -1);
    }
    pd.set(8, params[8]);
    int rc = chain->pack->load_param(pd);
    if (rc == 0)
        rc = chain->rope->load_param(pd);
    if (rc == 0)
        rc = chain->attention->load_param(pd);
    if (rc == 0)
        rc = chain->unpack->load_param(pd);
    *status = rc;
    chain->source_tokens = params[0] * params[1] * params[2];
    chain->text_tokens = params[6];
    chain->heads = heads;
    chain->head_dim = head_dim;
    chain->layout = layout;
    if (rc != 0)
    {
        delete chain;
        return nullptr;
    }
    return chain;
}

void ref_chain_destroy(void* handle)
{
    delete static_cast<RefChain*>(handle);
}

// Runs Pack -> MMRoPE -> WindowAttention -> Unpack on dense fp32 inputs.
// Each output pointer may be NULL. cu_seqlens receives the Pack's float blob.
// Returns the first non-zero layer status, else 0.
int ref_chain_forward(void* handle, const float* video_qkv, const float* text_qkv, float* packed, float* cu_seqlens,
                      float* roped, float* attended, float* video_out, float* text_out)
{
    RefChain* chain = static_cast<RefChain*>(handle);
    ncnn::Option opt;
    std::vector<ncnn::Mat> bottoms(2);
    if (!fill_qkv(bottoms[0], video_qkv, chain->source_tokens, chain->heads, chain->head_dim, chain->layout) ||
        !fill_qkv(bottoms[1], text_qkv, chain->text_tokens, chain->heads, chain->head_dim, chain->layout))
        return -1;

    std::vector<ncnn::Mat> pack_tops;
    double t0 = now_seconds();
    int rc = chain->pack->forward(bottoms, pack_tops, opt);
    double t1 = now_seconds();
    chain->seconds[0] = t1 - t0;
    if (rc != 0)
        return rc;
    if (packed)
        read_dense(pack_tops[0], packed);
    if (cu_seqlens)
        std::memcpy(cu_seqlens, pack_tops[1].data, sizeof(float) * pack_tops[1].w);

    std::vector<ncnn::Mat> rope_in(1, pack_tops[0]), rope_tops;
    t0 = now_seconds();
    rc = chain->rope->forward(rope_in, rope_tops, opt);
    t1 = now_seconds();
    chain->seconds[1] = t1 - t0;
    if (rc != 0)
        return rc;
    if (roped)
        read_dense(rope_tops[0], roped);

    std::vector<ncnn::Mat> attention_tops;
    t0 = now_seconds();
    rc = chain->attention->forward(rope_tops, attention_tops, opt);
    t1 = now_seconds();
    chain->seconds[2] = t1 - t0;
    if (rc != 0)
        return rc;
    if (attended)
        read_dense(attention_tops[0], attended);

    std::vector<ncnn::Mat> unpack_tops;
    t0 = now_seconds();
    rc = chain->unpack->forward(attention_tops, unpack_tops, opt);
    t1 = now_seconds();
    chain->seconds[3] = t1 - t0;
    if (rc != 0)
        return rc;
    if (video_out)
        read_dense(unpack_tops[0], video_out);
    if (text_out)
        read_dense(unpack_tops[1], text_out);
    return 0;
}

// Wall seconds of each layer's forward in the last ref_chain_forward call.
void ref_chain_seconds(void* handle, double* out4)
{
    RefChain* chain = static_cast<RefChain*>(handle);
    for (int i = 0; i < 4; i++)
        out4[i] = chain->seconds[i];
}

// Runs one layer alone on a dense input, for layer-level error checks.
// which: 0 pack (inputs video/text), 1 rope, 2 attention, 3 unpack.
int ref_layer_forward(void* handle, int which, const float* in0, const float* in1, int in_tokens, int in_rows,
                      float* out0, float* out1)
{
    RefChain* chain = static_cast<RefChain*>(handle);
    ncnn::Option opt;
    std::vector<ncnn::Mat> bottoms;
    ncnn::Layer* layer = which == 0 ? chain->pack : which == 1 ? chain->rope : which == 2 ? chain->attention
                                                                                         : chain->unpack;
    if (which == 0)
    {
        bottoms.resize(2);
        if (!fill_qkv(bottoms[0], in0, chain->source_tokens, chain->heads, chain->head_dim, chain->layout) ||
            !fill_qkv(bottoms[1], in1, chain->text_tokens, chain->heads, chain->head_dim, chain->layout))
            return -1;
    }
    else
    {
        bottoms.resize(1);
        bottoms[0].create(chain->head_dim, in_rows, in_tokens, 4u);
        const size_t plane = (size_t)chain->head_dim * in_rows;
        for (int t = 0; t < in_tokens; t++)
            std::memcpy(bottoms[0].channel(t).data, in0 + (size_t)t * plane, plane * sizeof(float));
    }
    std::vector<ncnn::Mat> tops;
    const int rc = layer->forward(bottoms, tops, opt);
    if (rc != 0)
        return rc;
    if (out0)
    {
        if (tops[0].dims == 1)
            std::memcpy(out0, tops[0].data, sizeof(float) * tops[0].w);
        else
            read_dense(tops[0], out0);
    }
    if (out1 && tops.size() > 1)
    {
        if (tops[1].dims == 1)
            std::memcpy(out1, tops[1].data, sizeof(float) * tops[1].w);
        else
            read_dense(tops[1], out1);
    }
    return 0;
}

} // extern "C"
