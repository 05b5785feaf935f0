// awa_rows.cuh -- where row r of window w lives, for the attention kernels.
//
// Window rows are the window's video tokens in (t, h, w) row-major order and
// then the text tokens: the order in which SeedVR2AWAPack lays them out
// (awa_layers.cpp:393-406). In packed mode a row is one packed token; in fused
// mode it is fetched directly from the source QKV by the window geometry, so
// the packed intermediate never exists.
#pragma once

#include "awa_device.cuh"
#include "awa_internal.h"

namespace awa
{

struct RowRef
{
    int64_t offset;   // element offset of the row's q segment of this head (qkv = 0)
    int64_t qkv_step; // elements between its q, k and v segments
    int is_text;      // fused mode: row comes from the text QKV
    int text_index;   // text token index when is_text
    int64_t token;    // fused mode, video rows: source token index
    short4 coords;    // RoPE coordinates (t, h, w) of the row
};

// Row `row` (< window length) of window `win` for head `head`.
template <bool PACKED>
__device__ __forceinline__ RowRef window_row(const AttnArgs& a, const WindowDesc& win, int row, int head)
{
    RowRef ref;
    const int text = a.plan.text_tokens;
    if (PACKED)
    {
        ref.offset = (int64_t)(win.offset + row) * a.qkv_token_stride + (int64_t)head * a.head_dim;
        ref.qkv_step = (int64_t)a.heads * a.head_dim;
        ref.is_text = row >= win.video;
        ref.text_index = row - win.video;
        ref.token = win.offset + row;
        ref.coords = make_short4(0, 0, 0, 0);
        return ref;
    }
    if (row < win.video)
    {
        const int plane = win.nh * win.nw;
        const int lt = row / plane;
        const int rem = row - lt * plane;
        const int lh = rem / win.nw;
        const int lw = rem - lh * win.nw;
        const int64_t token = ((int64_t)(win.t0 + lt) * a.plan.source_h + (win.h0 + lh)) * a.plan.source_w + (win.w0 + lw);
        ref.offset = token * a.video_token_stride + (int64_t)head * a.head_dim;
        ref.qkv_step = a.video_qkv_stride;
        ref.is_text = 0;
        ref.text_index = 0;
        ref.token = token;
        // window-local coordinates, t offset by the text count (awa_layers.cpp:906)
        ref.coords = make_short4((short)(text + lt), (short)lh, (short)lw, 0);
    }
    else
    {
        const int i = row - win.video;
        ref.offset = (int64_t)i * a.text_token_stride + (int64_t)head * a.head_dim;
        ref.qkv_step = a.text_qkv_stride;
        ref.is_text = 1;
        ref.text_index = i;
        ref.token = -1;
        ref.coords = make_short4((short)i, (short)i, (short)i, 0);  // awa_layers.cpp:907-908
    }
    return ref;
}

// Exact reference rotation (awa_layers.cpp:945-949): every product and the
// final sum/difference round separately (no FMA contraction).
__device__ __forceinline__ void rope_rotate(float x0, float x1, float c, float s, float& o0, float& o1)
{
    o0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    o1 = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
}

__device__ __forceinline__ float2 rope_lookup(const PlanDevice& plan, short4 coords, int pair)
{
    const int axis = pair / plan.pairs_per_axis;
    const int within = pair - axis * plan.pairs_per_axis;
    const int coord = axis == 0 ? coords.x : axis == 1 ? coords.y : coords.z;
    return __ldg(plan.rope_table + coord * plan.pairs_per_axis + within);
}

// Rotate 8 consecutive features starting at f (even) of a Q or K row.
__device__ __forceinline__ void rope8(const PlanDevice& plan, short4 coords, int f, float (&v)[8])
{
#pragma unroll
    for (int i = 0; i < 4; i++)
        if (f + 2 * i < plan.rope_dim)
        {
            const float2 cs = rope_lookup(plan, coords, (f >> 1) + i);
            rope_rotate(v[2 * i], v[2 * i + 1], cs.x, cs.y, v[2 * i], v[2 * i + 1]);
        }
}

// ex2.approx: 2^x (used for the softmax exponentials; |rel err| ~ 2^-22).
__device__ __forceinline__ float fast_exp2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

}  // namespace awa
