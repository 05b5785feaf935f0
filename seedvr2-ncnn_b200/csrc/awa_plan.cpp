// awa_plan.cpp -- host side of the B200 AWA layers: the window rule, index
// maps and RoPE table of a layer configuration (what the four ncnn layers
// build in load_param), their one-time upload, and the C ABI of
// include/awa_b200.h.
#include "awa_b200.h"
#include "awa_internal.h"

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <deque>
#include <limits>
#include <mutex>
#include <string>
#include <vector>

#include <cuda_runtime.h>

using awa::PlanDevice;
using awa::WindowDesc;

struct awa_plan
{
    awa_plan_info info{};
    int pairs_per_axis = 0;
    int max_coord = 0;
    std::vector<awa_window> windows;
    std::vector<WindowDesc> descs;
    std::vector<int> sequence_index;
    std::vector<int> cu_seqlens;
    std::vector<int> video_positions;
    std::vector<int> text_positions;
    std::vector<float2> rope_table;
    std::vector<uint2> rope_factors_bf16;  // per (coord, pair): bf16x2 (cos, cos), bf16x2 (-sin, sin)
    std::vector<short4> position_coords;
    std::vector<int2> items_tc;         // fused tcgen05 path: (window, pair of 128-row q tiles), longest first
    std::vector<int2> items_tc_packed;  // packed tcgen05 path: same, over the packed rows
    std::vector<int2> items_simt;       // (window, 128-row q tile)
    std::vector<double> window_cost;    // L^2 per window
    bool tc_slabs = false;              // every window is a clipped piece of a nominal-size window
    // device copies
    PlanDevice dev{};
    void* device_block = nullptr;
    const int2* d_items_tc = nullptr;
    const int2* d_items_tc_packed = nullptr;
    const int2* d_items_simt = nullptr;
    std::mutex range_mutex;  // guards the per-range and per-set caches below
    std::vector<std::pair<std::pair<int, int>, std::pair<int2*, int>>> range_items;  // (begin,end) -> items
    struct SetEntry
    {
        bool tc;
        std::vector<int> windows;  // sorted
        int2* items;               // device, the set's work items
        int count;
        int* slots;                // device [W]: slot of each window in the set, -1 outside
    };
    std::deque<SetEntry> set_items;  // a deque: entries stay put while others are added
};

namespace
{

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...)
{
    char buffer[512];
    va_list args;
    va_start(args, fmt);
    std::vsnprintf(buffer, sizeof(buffer), fmt, args);
    va_end(args);
    g_last_error = buffer;
    return code;
}

int cuda_fail(cudaError_t err, const char* what)
{
    return fail(err == cudaErrorMemoryAllocation ? AWA_ERR_ALLOC : AWA_ERR_CUDA, "%s: %s", what,
                cudaGetErrorString(err));
}

int ceil_div(int numerator, int denominator)
{
    return (numerator + denominator - 1) / denominator;
}

// Python round() (half to even) of a non-negative double: the window rule
// resizes the grid with it (awa_layers.cpp:41-51, seedvr2_baseline.py:45).
int round_half_even(double value)
{
    const double lower = std::floor(value);
    const double fraction = value - lower;
    if (fraction < 0.5)
        return static_cast<int>(lower);
    if (fraction > 0.5)
        return static_cast<int>(lower + 1.0);
    const int base = static_cast<int>(lower);
    return (base & 1) == 0 ? base : base + 1;
}

// The AWA window rule (awa_layers.cpp:53-88, seedvr2_baseline.py:37-79):
// the grid is rescaled to the area of a 45x80 grid, divided by the window
// counts (time capped at 30 frames), optionally shifted by half a window on
// every axis the window does not cover, clipped, and enumerated with w
// outermost and t innermost. Empty windows are dropped.
std::vector<awa_window> build_windows(int st, int sh, int sw, int nt, int nh, int nw, bool shifted)
{
    std::vector<awa_window> out;
    if (st <= 0 || sh <= 0 || sw <= 0 || nt <= 0 || nh <= 0 || nw <= 0)
        return out;
    const double area_scale = std::sqrt(3600.0 / (sh * sw));
    const int size_h = ceil_div(round_half_even(sh * area_scale), nh);
    const int size_w = ceil_div(round_half_even(sw * area_scale), nw);
    const int size_t_ = ceil_div(std::min(st, 30), nt);
    const double off_t = shifted && size_t_ < st ? 0.5 : 0.0;
    const double off_h = shifted && size_h < sh ? 0.5 : 0.0;
    const double off_w = shifted && size_w < sw ? 0.5 : 0.0;
    auto count = [](int extent, double off, int size) {
        return static_cast<int>(std::ceil((extent - off) / size)) + (off > 0 ? 1 : 0);
    };
    const int ct = count(st, off_t, size_t_), ch = count(sh, off_h, size_h), cw = count(sw, off_w, size_w);
    // (i - off) * size truncates toward zero before clipping, as the C++ cast does.
    auto lo = [](int i, double off, int size) { return std::max(static_cast<int>((i - off) * size), 0); };
    auto hi = [](int i, double off, int size, int extent) {
        return std::min(static_cast<int>((i - off + 1.0) * size), extent);
    };
    for (int iw = 0; iw < cw; iw++)
        for (int ih = 0; ih < ch; ih++)
            for (int it = 0; it < ct; it++)
            {
                awa_window win{lo(it, off_t, size_t_), hi(it, off_t, size_t_, st), lo(ih, off_h, size_h),
                               hi(ih, off_h, size_h, sh),   lo(iw, off_w, size_w),  hi(iw, off_w, size_w, sw)};
                if (win.t1 > win.t0 && win.h1 > win.h0 && win.w1 > win.w0)
                    out.push_back(win);
            }
    return out;
}

// Two floats rounded to bf16 (nearest even), packed low/high.
uint32_t bf16_pair(float lo, float hi)
{
    auto round = [](float f) -> uint32_t {
        uint32_t bits;
        std::memcpy(&bits, &f, 4);
        return (bits + 0x7fffu + ((bits >> 16) & 1u)) >> 16;
    };
    return round(lo) | (round(hi) << 16);
}

template <typename T>
size_t bytes_of(const std::vector<T>& v)
{
    return v.size() * sizeof(T);
}

size_t align_up(size_t v, size_t a)
{
    return (v + a - 1) / a * a;
}

bool valid_dtype(int dtype)
{
    return dtype == AWA_F32 || dtype == AWA_BF16;
}

size_t dtype_size(int dtype)
{
    return dtype == AWA_F32 ? 4 : 2;
}

int check_device(const awa_plan* plan)
{
    if (!plan->device_block)
        return fail(AWA_ERR_INVALID, "plan was created without device tables (awa_plan_create_host)");
    int device = -1;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess)
        return cuda_fail(err, "cudaGetDevice");
    if (device != plan->info.device)
        return fail(AWA_ERR_INVALID, "plan lives on device %d but device %d is current", plan->info.device, device);
    return AWA_OK;
}

int check_heads(const awa_plan* plan, int heads, int head_dim)
{
    if (!plan)
        return fail(AWA_ERR_INVALID, "plan is NULL");
    if (heads <= 0 || head_dim <= 0)
        return fail(AWA_ERR_INVALID, "heads (%d) and head_dim (%d) must be positive", heads, head_dim);
    if (head_dim > awa::kMaxHeadDim)
        return fail(AWA_ERR_INVALID, "head_dim %d exceeds the supported maximum %d", head_dim, awa::kMaxHeadDim);
    if ((int64_t)plan->info.sequence_tokens * 3 * heads * head_dim > std::numeric_limits<int64_t>::max() / 4)
        return fail(AWA_ERR_INVALID, "problem too large");
    return check_device(plan);
}

int launch_status(int err, const char* what)
{
    if (err != cudaSuccess)
        return cuda_fail(static_cast<cudaError_t>(err), what);
    return AWA_OK;
}

}  // namespace

namespace awa
{

int report_error(int code, const char* message)
{
    return fail(code, "%s", message);
}

int* device_error_flag()
{
    static std::mutex mutex;
    static int* flags[64] = {nullptr};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64)
        return nullptr;
    std::lock_guard<std::mutex> lock(mutex);
    if (!flags[device])
    {
        int* p = nullptr;
        if (cudaMalloc(&p, sizeof(int)) != cudaSuccess)
            return nullptr;
        if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess)
            return nullptr;
        flags[device] = p;
    }
    return flags[device];
}

}  // namespace awa

extern "C" {

const char* awa_last_error(void)
{
    return g_last_error.c_str();
}

const char* awa_version(void)
{
    return "seedvr2-awa-b200 0.1 (sm_100a)";
}

int awa_make_windows(int source_t, int source_h, int source_w, int windows_t, int windows_h, int windows_w,
                     int shifted, awa_window* out, int capacity)
{
    const std::vector<awa_window> windows =
        build_windows(source_t, source_h, source_w, windows_t, windows_h, windows_w, shifted != 0);
    if (out)
        for (size_t i = 0; i < windows.size() && static_cast<int>(i) < capacity; i++)
            out[i] = windows[i];
    return static_cast<int>(windows.size());
}

static int plan_create_impl(const awa_layer_params* params, const awa_runtime_spec* spec, awa_plan** out_plan,
                            bool upload)
{
    if (!params || !out_plan)
        return fail(AWA_ERR_INVALID, "params and out_plan must not be NULL");
    *out_plan = nullptr;
    int st = params->source_t, sh = params->source_h, sw = params->source_w;
    // load_common (awa_layers.cpp:90-114): -1,-1,-1 takes the grid from the runtime spec.
    if (st == -1 && sh == -1 && sw == -1)
    {
        const long long tokens = spec ? (long long)spec->source_t * spec->source_h * spec->source_w : 0;
        if (!spec || spec->source_t <= 0 || spec->source_h <= 0 || spec->source_w <= 0 || spec->video_tokens <= 0 ||
            tokens != spec->video_tokens || tokens > std::numeric_limits<int>::max())
            return fail(AWA_ERR_INVALID, "grid is -1,-1,-1 but the runtime spec is missing or invalid");
        st = spec->source_t;
        sh = spec->source_h;
        sw = spec->source_w;
    }
    const long long source_tokens = (long long)st * sh * sw;
    if (st <= 0 || sh <= 0 || sw <= 0 || params->windows_t <= 0 || params->windows_h <= 0 ||
        params->windows_w <= 0 || params->text_tokens <= 0 || source_tokens > std::numeric_limits<int>::max())
        return fail(AWA_ERR_INVALID, "invalid AWA params %d %d %d / %d %d %d / text %d", st, sh, sw,
                    params->windows_t, params->windows_h, params->windows_w, params->text_tokens);
    const int rope_dim = params->rope_dim == 0 ? 126 : params->rope_dim;
    if (rope_dim <= 0 || rope_dim % 6 != 0)  // awa_layers.cpp:872-874
        return fail(AWA_ERR_INVALID, "rope_dim %d must be a positive multiple of 6", rope_dim);
    const int text = params->text_tokens;

    awa_plan* plan = new (std::nothrow) awa_plan();
    if (!plan)
        return fail(AWA_ERR_ALLOC, "out of host memory");
    plan->windows = build_windows(st, sh, sw, params->windows_t, params->windows_h, params->windows_w,
                                  params->shifted != 0);
    const int window_count = static_cast<int>(plan->windows.size());
    long long sequence = source_tokens + (long long)window_count * text;
    if (window_count == 0 || sequence > std::numeric_limits<int>::max() / 4)
    {
        delete plan;
        return fail(AWA_ERR_INVALID, "window layout is empty or too large");
    }
    const int S = static_cast<int>(sequence);

    // Index maps (awa_layers.cpp:388-407 Pack, 605-626 Unpack, 1051-1058 attention).
    plan->sequence_index.reserve(S);
    plan->cu_seqlens.reserve(window_count + 1);
    plan->video_positions.assign(source_tokens, -1);
    plan->text_positions.reserve((size_t)window_count * text);
    plan->position_coords.reserve(S);
    plan->cu_seqlens.push_back(0);
    int max_length = 0;
    int max_coord = text;
    for (const awa_window& win : plan->windows)
    {
        WindowDesc desc;
        desc.t0 = win.t0;
        desc.h0 = win.h0;
        desc.w0 = win.w0;
        desc.nt = win.t1 - win.t0;
        desc.nh = win.h1 - win.h0;
        desc.nw = win.w1 - win.w0;
        desc.offset = static_cast<int>(plan->sequence_index.size());
        desc.video = desc.nt * desc.nh * desc.nw;
        plan->descs.push_back(desc);
        for (int t = win.t0; t < win.t1; t++)
            for (int h = win.h0; h < win.h1; h++)
                for (int w = win.w0; w < win.w1; w++)
                {
                    const int source = (t * sh + h) * sw + w;
                    if (plan->video_positions[source] != -1)
                    {
                        delete plan;
                        return fail(AWA_ERR_INVALID, "token %d is covered by two windows", source);
                    }
                    plan->video_positions[source] = static_cast<int>(plan->sequence_index.size());
                    plan->sequence_index.push_back(source);
                    // RoPE coordinates of a video token: window-local, t offset by the
                    // text count (awa_layers.cpp:906).
                    plan->position_coords.push_back(make_short4((short)(text + t - win.t0), (short)(h - win.h0),
                                                                (short)(w - win.w0), 0));
                }
        for (int i = 0; i < text; i++)
        {
            plan->text_positions.push_back(static_cast<int>(plan->sequence_index.size()));
            plan->sequence_index.push_back(static_cast<int>(source_tokens) + i);
            plan->position_coords.push_back(make_short4((short)i, (short)i, (short)i, 0));  // :907-908
        }
        plan->cu_seqlens.push_back(static_cast<int>(plan->sequence_index.size()));
        const int length = desc.video + text;
        max_length = std::max(max_length, length);
        max_coord = std::max({max_coord, text + desc.nt, desc.nh, desc.nw});
        plan->window_cost.push_back((double)length * length);
    }
    for (int v : plan->video_positions)
        if (v < 0)
        {
            delete plan;
            return fail(AWA_ERR_INVALID, "window layout does not cover every token");  // awa_layers.cpp:635
        }
    if (max_coord > 32767)
    {
        delete plan;
        return fail(AWA_ERR_INVALID, "window too large for the RoPE coordinate table");
    }

    // RoPE table: only (coordinate, pair) matters, because the reference's
    // per-position table (awa_layers.cpp:884-898) holds cos/sin of
    // coordinate * powf(10000, -2p/axis_dim) for each axis. Same float
    // expressions, so every entry is bit-identical to the reference's.
    plan->pairs_per_axis = rope_dim / 6;
    plan->max_coord = max_coord;
    const int axis_dim = rope_dim / 3;
    plan->rope_table.resize((size_t)max_coord * plan->pairs_per_axis);
    // factor rows padded to an even length, so two pairs of one axis starting at
    // an even pair load as one 16-byte vector
    const int factor_stride = plan->pairs_per_axis + (plan->pairs_per_axis & 1);
    plan->rope_factors_bf16.assign((size_t)max_coord * factor_stride, make_uint2(0u, 0u));
    for (int pair = 0; pair < plan->pairs_per_axis; pair++)
    {
        const float frequency = std::pow(10000.f, -static_cast<float>(2 * pair) / axis_dim);
        for (int coord = 0; coord < max_coord; coord++)
        {
            const float angle = coord * frequency;
            const float c = std::cos(angle), sn = std::sin(angle);
            plan->rope_table[(size_t)coord * plan->pairs_per_axis + pair] = make_float2(c, sn);
            // the tensor-core kernel's rotation factors of the same entry, in bf16:
            // x' = x c - y s, y' = y c + x s as (x, y) * (c, c) + (y, x) * (-s, s)
            const uint32_t cs = bf16_pair(c, sn);
            const uint32_t cc = (cs & 0xffffu) | (cs << 16);
            const uint32_t ns = ((cs >> 16) | (cs & 0xffff0000u)) ^ 0x8000u;
            plan->rope_factors_bf16[(size_t)coord * factor_stride + pair] = make_uint2(cc, ns);
        }
    }

    // Slab geometry of the tcgen05 kernel. The window rule tiles each axis
    // with windows of one nominal size, clipped only at the grid's edges, so
    // laying a nominal-size box over each window reads nothing of another
    // window: the part of the box outside the window lies outside the grid.
    // Checked for every window; without it the SIMT kernel runs.
    {
        int bh = 0, bw = 0;
        for (const WindowDesc& d : plan->descs)
        {
            bh = std::max(bh, d.nh);
            bw = std::max(bw, d.nw);
        }
        auto nominal_start = [](int start, int count, int size) { return start == 0 ? start + count - size : start; };
        bool ok = true;
        for (WindowDesc& d : plan->descs)
        {
            d.h0n = nominal_start(d.h0, d.nh, bh);
            d.w0n = nominal_start(d.w0, d.nw, bw);
            // the box [x0n, x0n + size) clipped to the grid must be exactly the window
            ok = ok && std::max(d.h0n, 0) == d.h0 && std::min(d.h0n + bh, sh) == d.h0 + d.nh &&
                 std::max(d.w0n, 0) == d.w0 && std::min(d.w0n + bw, sw) == d.w0 + d.nw;
        }
        PlanDevice& g = plan->dev;
        g.tc_bh = bh;
        g.tc_bw = bw;
        g.tc_bwc = std::min(bw, 64);
        g.tc_bhc = std::max(1, std::min(bh, 64 / g.tc_bwc));
        g.tc_nhc = ceil_div(bh, g.tc_bhc);
        g.tc_nwc = ceil_div(bw, g.tc_bwc);
        g.tc_rows = g.tc_bhc * g.tc_bwc;
        g.tc_text_blocks = ceil_div(text, 64);
        plan->tc_slabs = ok && bh <= 256 && bw <= 256;
    }

    // Work lists, longest windows first so the tail of the grid is short.
    // tcgen05 items are pairs of 128-row query tiles = 4 key blocks of 64 rows.
    std::vector<int> order(window_count);
    for (int i = 0; i < window_count; i++)
        order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return plan->window_cost[a] > plan->window_cost[b]; });
    const PlanDevice& g = plan->dev;
    for (int w : order)
    {
        const WindowDesc& d = plan->descs[w];
        const int length = d.video + text;
        const int fused_blocks = d.nt * g.tc_nhc * g.tc_nwc + g.tc_text_blocks;
        for (int q = 0; q < ceil_div(fused_blocks, 4); q++)
            plan->items_tc.push_back(make_int2(w, q));
        for (int q = 0; q < ceil_div(length, 4 * 64); q++)
            plan->items_tc_packed.push_back(make_int2(w, q));
        for (int q = 0; q < ceil_div(length, awa::kSimtRowsPerTile); q++)
            plan->items_simt.push_back(make_int2(w, q));
    }

    plan->info.source_t = st;
    plan->info.source_h = sh;
    plan->info.source_w = sw;
    plan->info.source_tokens = static_cast<int>(source_tokens);
    plan->info.text_tokens = text;
    plan->info.window_count = window_count;
    plan->info.sequence_tokens = S;
    plan->info.max_window_length = max_length;
    plan->info.rope_dim = rope_dim;
    plan->info.shifted = params->shifted != 0;

    if (!upload)
    {
        plan->info.device = -1;
        *out_plan = plan;
        return AWA_OK;
    }
    // One device block holds every table.
    cudaError_t err = cudaGetDevice(&plan->info.device);
    if (err != cudaSuccess)
    {
        delete plan;
        return cuda_fail(err, "cudaGetDevice");
    }
    constexpr int kSegments = 10;
    size_t offsets[kSegments];
    size_t total = 0;
    const size_t sizes[kSegments] = {
        bytes_of(plan->descs),           bytes_of(plan->sequence_index), bytes_of(plan->cu_seqlens),
        bytes_of(plan->video_positions), bytes_of(plan->position_coords), bytes_of(plan->rope_table),
        bytes_of(plan->items_tc),        bytes_of(plan->items_simt),      bytes_of(plan->rope_factors_bf16),
        bytes_of(plan->items_tc_packed)};
    for (int i = 0; i < kSegments; i++)
    {
        offsets[i] = total;
        total = align_up(total + sizes[i], 256);
    }
    err = cudaMalloc(&plan->device_block, total);
    if (err != cudaSuccess)
    {
        delete plan;
        return cuda_fail(err, "cudaMalloc(plan tables)");
    }
    std::vector<unsigned char> staging(total, 0);
    const void* sources[kSegments] = {
        plan->descs.data(),           plan->sequence_index.data(),  plan->cu_seqlens.data(),
        plan->video_positions.data(), plan->position_coords.data(), plan->rope_table.data(),
        plan->items_tc.data(),        plan->items_simt.data(),      plan->rope_factors_bf16.data(),
        plan->items_tc_packed.data()};
    for (int i = 0; i < kSegments; i++)
        if (sizes[i])
            std::memcpy(staging.data() + offsets[i], sources[i], sizes[i]);
    err = cudaMemcpy(plan->device_block, staging.data(), total, cudaMemcpyHostToDevice);
    if (err != cudaSuccess)
    {
        cudaFree(plan->device_block);
        delete plan;
        return cuda_fail(err, "cudaMemcpy(plan tables)");
    }
    unsigned char* base = static_cast<unsigned char*>(plan->device_block);
    PlanDevice& dev = plan->dev;
    dev.windows = reinterpret_cast<const WindowDesc*>(base + offsets[0]);
    dev.sequence_index = reinterpret_cast<const int*>(base + offsets[1]);
    dev.cu_seqlens = reinterpret_cast<const int*>(base + offsets[2]);
    dev.video_positions = reinterpret_cast<const int*>(base + offsets[3]);
    dev.position_coords = reinterpret_cast<const int*>(base + offsets[4]);
    dev.rope_table = reinterpret_cast<const float2*>(base + offsets[5]);
    dev.rope_factors_bf16 = reinterpret_cast<const uint2*>(base + offsets[8]);
    plan->d_items_tc = reinterpret_cast<const int2*>(base + offsets[6]);
    plan->d_items_simt = reinterpret_cast<const int2*>(base + offsets[7]);
    plan->d_items_tc_packed = reinterpret_cast<const int2*>(base + offsets[9]);
    dev.source_t = st;
    dev.source_h = sh;
    dev.source_w = sw;
    dev.source_tokens = static_cast<int>(source_tokens);
    dev.text_tokens = text;
    dev.window_count = window_count;
    dev.sequence_tokens = S;
    dev.rope_dim = rope_dim;
    dev.pairs_per_axis = plan->pairs_per_axis;
    dev.max_coord = max_coord;
    dev.max_window_video = max_length - text;
    if (!awa::device_error_flag())
    {
        cudaFree(plan->device_block);
        delete plan;
        return fail(AWA_ERR_ALLOC, "could not allocate the device status flag");
    }
    *out_plan = plan;
    return AWA_OK;
}

int awa_plan_create(const awa_layer_params* params, const awa_runtime_spec* spec, awa_plan** out_plan)
{
    return plan_create_impl(params, spec, out_plan, true);
}

int awa_plan_create_host(const awa_layer_params* params, const awa_runtime_spec* spec, awa_plan** out_plan)
{
    return plan_create_impl(params, spec, out_plan, false);
}

void awa_plan_destroy(awa_plan* plan)
{
    if (!plan)
        return;
    if (plan->device_block)
    {
        for (auto& entry : plan->range_items)
            cudaFree(entry.second.first);
        for (auto& entry : plan->set_items)
        {
            cudaFree(entry.items);
            cudaFree(entry.slots);
        }
        cudaFree(plan->device_block);
    }
    delete plan;
}

int awa_plan_get_info(const awa_plan* plan, awa_plan_info* info)
{
    if (!plan || !info)
        return fail(AWA_ERR_INVALID, "plan and info must not be NULL");
    *info = plan->info;
    return AWA_OK;
}

int awa_plan_get_maps(const awa_plan* plan, int* sequence_index, int* cu_seqlens, int* video_positions,
                      int* text_positions, awa_window* windows)
{
    if (!plan)
        return fail(AWA_ERR_INVALID, "plan is NULL");
    if (sequence_index)
        std::memcpy(sequence_index, plan->sequence_index.data(), bytes_of(plan->sequence_index));
    if (cu_seqlens)
        std::memcpy(cu_seqlens, plan->cu_seqlens.data(), bytes_of(plan->cu_seqlens));
    if (video_positions)
        std::memcpy(video_positions, plan->video_positions.data(), bytes_of(plan->video_positions));
    if (text_positions)
        std::memcpy(text_positions, plan->text_positions.data(), bytes_of(plan->text_positions));
    if (windows)
        std::memcpy(windows, plan->windows.data(), bytes_of(plan->windows));
    return AWA_OK;
}

int awa_pack(const awa_plan* plan, int heads, int head_dim, int in_dtype, const void* video_qkv,
             int64_t video_token_stride, int64_t video_qkv_stride, const void* text_qkv, int64_t text_token_stride,
             int64_t text_qkv_stride, int out_dtype, void* packed, int64_t packed_token_stride, float* cu_seqlens,
             awa_stream_t stream)
{
    int rc = check_heads(plan, heads, head_dim);
    if (rc)
        return rc;
    const int64_t head_row = (int64_t)heads * head_dim;
    if (!valid_dtype(in_dtype) || !valid_dtype(out_dtype) || !video_qkv || !text_qkv || !packed)
        return fail(AWA_ERR_INVALID, "awa_pack: invalid dtype or NULL tensor");
    if (video_qkv_stride < head_row || text_qkv_stride < head_row || video_token_stride < head_row ||
        text_token_stride < head_row || packed_token_stride < 3 * head_row)
        return fail(AWA_ERR_INVALID, "awa_pack: strides smaller than a row");
    return launch_status(awa::launch_pack(plan->dev, heads, head_dim, in_dtype, video_qkv, video_token_stride,
                                          video_qkv_stride, text_qkv, text_token_stride, text_qkv_stride, out_dtype,
                                          packed, packed_token_stride, cu_seqlens, stream),
                         "awa_pack launch");
}

int awa_mmrope(const awa_plan* plan, int heads, int head_dim, int in_dtype, const void* packed_in,
               int64_t in_token_stride, int out_dtype, void* packed_out, int64_t out_token_stride,
               awa_stream_t stream)
{
    int rc = check_heads(plan, heads, head_dim);
    if (rc)
        return rc;
    if (!valid_dtype(in_dtype) || !valid_dtype(out_dtype) || !packed_in || !packed_out)
        return fail(AWA_ERR_INVALID, "awa_mmrope: invalid dtype or NULL tensor");
    if (head_dim < plan->info.rope_dim)  // awa_layers.cpp:920
        return fail(AWA_ERR_INVALID, "awa_mmrope: head_dim %d < rope_dim %d", head_dim, plan->info.rope_dim);
    const int64_t row = 3LL * heads * head_dim;
    if (in_token_stride < row || out_token_stride < row)
        return fail(AWA_ERR_INVALID, "awa_mmrope: strides smaller than a row");
    return launch_status(awa::launch_mmrope(plan->dev, heads, head_dim, in_dtype, packed_in, in_token_stride,
                                            out_dtype, packed_out, out_token_stride, stream),
                         "awa_mmrope launch");
}

// The tcgen05 kernel serves bf16 blocks with head_dim 128 on plans whose
// windows it can fetch as boxes. It reads bf16 rows; the fused forward
// converts fp32 QKV rows to bf16 into its workspace first.
static bool tc_capable(const awa_plan* plan, int precision, int head_dim)
{
    return plan && precision == AWA_PREC_BF16 && head_dim == 128 && plan->tc_slabs;
}

int awa_attention_kernel_kind(const awa_plan* plan, int precision, int in_dtype, int heads, int head_dim)
{
    (void)heads;
    (void)in_dtype;
    return tc_capable(plan, precision, head_dim) ? 1 : 2;
}

// Bytes of the bf16 copy of the QKV rows that the fused forward makes for
// fp32 rows on the tensor-core path (video then text, 256-byte aligned).
static size_t conversion_bytes(const awa_plan* plan, int heads, int head_dim)
{
    const size_t row = 3 * (size_t)heads * head_dim * 2;
    auto a256 = [](size_t v) { return (v + 255) & ~(size_t)255; };
    return a256((size_t)plan->info.source_tokens * row) + a256((size_t)plan->info.text_tokens * row);
}

static int run_attention(const awa_plan* plan, int precision, awa::AttnArgs& args, int packed, int in_dtype,
                         int out_dtype, const int2* items, int item_count, cudaStream_t stream)
{
    args.plan = plan->dev;
    args.scale = 1.f / std::sqrt(static_cast<float>(args.head_dim));
    args.error_flag = awa::device_error_flag();
    args.items = items;
    args.item_count = item_count;
    if (item_count == 0)
        return AWA_OK;
    if (tc_capable(plan, precision, args.head_dim) && in_dtype == AWA_BF16)
        return launch_status(awa::launch_attention_tc(args, packed, in_dtype, out_dtype, stream), "tcgen05 attention");
    return launch_status(awa::launch_attention_simt(args, packed, in_dtype, out_dtype, stream), "simt attention");
}

static bool is_aligned16(const void* p)
{
    return (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

int awa_window_attention(const awa_plan* plan, int precision, int heads, int head_dim, int in_dtype,
                         const void* packed, int64_t in_token_stride, int out_dtype, void* attended,
                         int64_t out_token_stride, awa_stream_t stream)
{
    int rc = check_heads(plan, heads, head_dim);
    if (rc)
        return rc;
    if (!valid_dtype(in_dtype) || !valid_dtype(out_dtype) || !packed || !attended ||
        (precision != AWA_PREC_FP32 && precision != AWA_PREC_BF16))
        return fail(AWA_ERR_INVALID, "awa_window_attention: invalid dtype/precision or NULL tensor");
    if (in_token_stride < 3LL * heads * head_dim || out_token_stride < (int64_t)heads * head_dim)
        return fail(AWA_ERR_INVALID, "awa_window_attention: strides smaller than a row");
    awa::AttnArgs args;
    args.heads = heads;
    args.head_dim = head_dim;
    args.qkv = packed;
    args.qkv_token_stride = in_token_stride;
    args.out = attended;
    args.out_token_stride = out_token_stride;
    const bool tc = tc_capable(plan, precision, head_dim) && in_dtype == AWA_BF16;  // packed rows: bf16 only
    if (tc && (!is_aligned16(packed) || !is_aligned16(attended) || (in_token_stride * dtype_size(in_dtype)) % 16 ||
               (out_token_stride * dtype_size(out_dtype)) % 16))
        return fail(AWA_ERR_INVALID, "awa_window_attention: bf16 tensor-core path needs 16-byte aligned rows");
    return run_attention(plan, precision, args, 1, in_dtype, out_dtype,
                         tc ? plan->d_items_tc_packed : plan->d_items_simt,
                         static_cast<int>(tc ? plan->items_tc_packed.size() : plan->items_simt.size()), stream);
}

int awa_unpack(const awa_plan* plan, int heads, int head_dim, int in_dtype, const void* attended,
               int64_t in_token_stride, int out_dtype, void* video_out, int64_t video_token_stride,
               void* text_out, int64_t text_token_stride, awa_stream_t stream)
{
    int rc = check_heads(plan, heads, head_dim);
    if (rc)
        return rc;
    const int64_t row = (int64_t)heads * head_dim;
    if (!valid_dtype(in_dtype) || !valid_dtype(out_dtype) || !attended || !video_out || !text_out)
        return fail(AWA_ERR_INVALID, "awa_unpack: invalid dtype or NULL tensor");
    if (in_token_stride < row || video_token_stride < row || text_token_stride < row)
        return fail(AWA_ERR_INVALID, "awa_unpack: strides smaller than a row");
    rc = launch_status(awa::launch_unpack_video(plan->dev, heads, head_dim, in_dtype, attended, in_token_stride,
                                                out_dtype, video_out, video_token_stride, stream),
                       "awa_unpack video launch");
    if (rc)
        return rc;
    return launch_status(awa::launch_text_reduce(plan->dev, heads, head_dim, 1, in_dtype, attended, in_token_stride, 0,
                                                 plan->info.window_count, (float)plan->info.window_count, out_dtype,
                                                 text_out, text_token_stride, stream),
                         "awa_unpack text launch");
}

size_t awa_forward_workspace_bytes(const awa_plan* plan, int heads, int head_dim)
{
    if (!plan || heads <= 0 || head_dim <= 0)
        return 0;
    return (size_t)plan->info.window_count * plan->info.text_tokens * heads * head_dim * sizeof(float);
}

size_t awa_forward_workspace_bytes_for(const awa_plan* plan, int precision, int in_dtype, int heads, int head_dim)
{
    const size_t base = awa_forward_workspace_bytes(plan, heads, head_dim);
    if (base == 0 || !(tc_capable(plan, precision, head_dim) && in_dtype == AWA_F32))
        return base;
    return ((base + 255) & ~(size_t)255) + conversion_bytes(plan, heads, head_dim);
}

// Items of windows [begin, end) in work order; cached per range on the device.
static const int2* range_items(awa_plan* plan, bool tc, int begin, int end, int* count, int* rc)
{
    *rc = AWA_OK;
    if (begin == 0 && end == plan->info.window_count)
    {
        *count = static_cast<int>(tc ? plan->items_tc.size() : plan->items_simt.size());
        return tc ? plan->d_items_tc : plan->d_items_simt;
    }
    std::lock_guard<std::mutex> lock(plan->range_mutex);
    const int key_begin = tc ? begin : -1 - begin;
    for (auto& entry : plan->range_items)
        if (entry.first.first == key_begin && entry.first.second == end)
        {
            *count = entry.second.second;
            return entry.second.first;
        }
    std::vector<int2> items;
    for (const int2& item : tc ? plan->items_tc : plan->items_simt)
        if (item.x >= begin && item.x < end)
            items.push_back(item);
    int2* d = nullptr;
    if (!items.empty())
    {
        cudaError_t err = cudaMalloc(&d, bytes_of(items));
        if (err == cudaSuccess)
            err = cudaMemcpy(d, items.data(), bytes_of(items), cudaMemcpyHostToDevice);
        if (err != cudaSuccess)
        {
            *rc = cuda_fail(err, "range work list");
            return nullptr;
        }
    }
    plan->range_items.push_back({{key_begin, end}, {d, static_cast<int>(items.size())}});
    *count = static_cast<int>(items.size());
    return d;
}

// Items and slot map of a window set (sorted, distinct), cached on the device.
static const awa_plan::SetEntry* set_items(awa_plan* plan, bool tc, const int* windows, int n, int* rc)
{
    *rc = AWA_OK;
    std::vector<int> key(windows, windows + n);
    std::lock_guard<std::mutex> lock(plan->range_mutex);
    for (const auto& e : plan->set_items)
        if (e.tc == tc && e.windows == key)
            return &e;
    const int W = plan->info.window_count;
    std::vector<int> slots(W, -1);
    for (int k = 0; k < n; k++)
    {
        if (windows[k] < 0 || windows[k] >= W || (k > 0 && windows[k] <= windows[k - 1]))
        {
            *rc = fail(AWA_ERR_INVALID, "window set: indices must be sorted, distinct and < %d", W);
            return nullptr;
        }
        slots[windows[k]] = k;
    }
    std::vector<int2> items;
    for (const int2& item : tc ? plan->items_tc : plan->items_simt)
        if (slots[item.x] >= 0)
            items.push_back(item);
    awa_plan::SetEntry e{tc, key, nullptr, (int)items.size(), nullptr};
    cudaError_t err = cudaMalloc(&e.slots, bytes_of(slots));
    if (err == cudaSuccess)
        err = cudaMemcpy(e.slots, slots.data(), bytes_of(slots), cudaMemcpyHostToDevice);
    if (err == cudaSuccess && !items.empty())
        err = cudaMalloc(&e.items, bytes_of(items));
    if (err == cudaSuccess && !items.empty())
        err = cudaMemcpy(e.items, items.data(), bytes_of(items), cudaMemcpyHostToDevice);
    if (err != cudaSuccess)
    {
        cudaFree(e.slots);
        cudaFree(e.items);
        *rc = cuda_fail(err, "window set work list");
        return nullptr;
    }
    plan->set_items.push_back(std::move(e));
    return &plan->set_items.back();
}

// Runs the fused attention over windows [window_begin, window_end); the text
// rows' per-window outputs go to the workspace as partials of *partial_dtype
// (bf16 from the tensor-core kernel, as the layer chain's bf16 attended rows;
// fp32 from the SIMT kernel).
static int forward_impl(const awa_plan* cplan, int precision, int heads, int head_dim, int window_begin,
                        int window_end, int in_dtype, const void* video_qkv, int64_t vts, int64_t vqs,
                        const void* text_qkv, int64_t tts, int64_t tqs, int out_dtype, void* video_out,
                        int64_t vots, void* workspace, size_t workspace_bytes, int* partial_dtype,
                        cudaStream_t stream, int rotate = 1, const int* window_set = nullptr, int set_count = 0)
{
    awa_plan* plan = const_cast<awa_plan*>(cplan);
    const int64_t head_row = (int64_t)heads * head_dim;
    if (!valid_dtype(in_dtype) || !valid_dtype(out_dtype) || !video_qkv || !text_qkv || !video_out ||
        (precision != AWA_PREC_FP32 && precision != AWA_PREC_BF16))
        return fail(AWA_ERR_INVALID, "awa_forward: invalid dtype/precision or NULL tensor");
    if (vqs < head_row || tqs < head_row || vts < head_row || tts < head_row || vots < head_row)
        return fail(AWA_ERR_INVALID, "awa_forward: strides smaller than a row");
    if (head_dim < plan->info.rope_dim)
        return fail(AWA_ERR_INVALID, "awa_forward: head_dim %d < rope_dim %d", head_dim, plan->info.rope_dim);
    const size_t need = (size_t)(window_set ? set_count : window_end - window_begin) * plan->info.text_tokens *
                        head_row * sizeof(float);
    if (!workspace || workspace_bytes < need)
        return fail(AWA_ERR_INVALID, "awa_forward: workspace of %zu bytes needed, %zu given", need, workspace_bytes);
    const bool tc = tc_capable(plan, precision, head_dim);
    *partial_dtype = tc ? AWA_BF16 : AWA_F32;
    if (tc && in_dtype == AWA_F32)
    {
        // fp32 rows (a bf16 block fed the reference's promoted fp32 QKV,
        // dit_precision.cpp:314-315): one pass converts them to dense bf16 rows
        // in the workspace behind the text partials; the kernel reads those.
        const size_t at = (need + 255) & ~(size_t)255;
        const size_t total = at + conversion_bytes(plan, heads, head_dim);
        if (workspace_bytes < total)
            return fail(AWA_ERR_INVALID,
                        "awa_forward: fp32 QKV on the tensor-core path needs a workspace of %zu bytes "
                        "(awa_forward_workspace_bytes_for), %zu given",
                        total, workspace_bytes);
        unsigned char* vdst = static_cast<unsigned char*>(workspace) + at;
        unsigned char* tdst = vdst + (((size_t)plan->info.source_tokens * 3 * head_row * 2 + 255) & ~(size_t)255);
        int rc = launch_status(awa::launch_rows_to_bf16(video_qkv, vts, vqs, plan->info.source_tokens, head_row, vdst,
                                                        stream),
                               "awa_forward fp32 -> bf16 rows (video)");
        if (rc == AWA_OK)
            rc = launch_status(awa::launch_rows_to_bf16(text_qkv, tts, tqs, plan->info.text_tokens, head_row, tdst,
                                                        stream),
                               "awa_forward fp32 -> bf16 rows (text)");
        if (rc)
            return rc;
        video_qkv = vdst;
        text_qkv = tdst;
        vts = tts = 3 * head_row;
        vqs = tqs = head_row;
        in_dtype = AWA_BF16;
    }
    if (tc)
    {
        const size_t in_size = dtype_size(in_dtype), out_size = dtype_size(out_dtype);
        if (!is_aligned16(video_qkv) || !is_aligned16(text_qkv) || !is_aligned16(video_out) ||
            (vts * in_size) % 16 || (vqs * in_size) % 16 || (tts * in_size) % 16 || (tqs * in_size) % 16 ||
            (vots * out_size) % 16)
            return fail(AWA_ERR_INVALID, "awa_forward: bf16 tensor-core path needs 16-byte aligned rows");
    }
    awa::AttnArgs args;
    args.heads = heads;
    args.head_dim = head_dim;
    args.video_qkv = video_qkv;
    args.video_token_stride = vts;
    args.video_qkv_stride = vqs;
    args.text_qkv = text_qkv;
    args.text_token_stride = tts;
    args.text_qkv_stride = tqs;
    args.out = video_out;
    args.out_token_stride = vots;
    args.text_partial = static_cast<float*>(workspace);
    args.window_begin = window_begin;
    args.rotate = rotate;
    int count = 0, rc = AWA_OK;
    const int2* items = nullptr;
    if (window_set)
    {
        const awa_plan::SetEntry* e = set_items(plan, tc, window_set, set_count, &rc);
        if (rc)
            return rc;
        items = e->items;
        count = e->count;
        args.partial_slot = e->slots;
    }
    else
        items = range_items(plan, tc, window_begin, window_end, &count, &rc);
    if (rc)
        return rc;
    return run_attention(plan, precision, args, 0, in_dtype, out_dtype, items, count, stream);
}

static int forward_whole(const awa_plan* plan, int precision, int heads, int head_dim, int in_dtype,
                         const void* video_qkv, int64_t video_token_stride, int64_t video_qkv_stride,
                         const void* text_qkv, int64_t text_token_stride, int64_t text_qkv_stride, int out_dtype,
                         void* video_out, int64_t video_token_stride_out, void* text_out,
                         int64_t text_token_stride_out, void* workspace, size_t workspace_bytes, awa_stream_t stream,
                         int rotate);

int awa_forward(const awa_plan* plan, int precision, int heads, int head_dim, int in_dtype, const void* video_qkv,
                int64_t video_token_stride, int64_t video_qkv_stride, const void* text_qkv,
                int64_t text_token_stride, int64_t text_qkv_stride, int out_dtype, void* video_out,
                int64_t video_token_stride_out, void* text_out, int64_t text_token_stride_out, void* workspace,
                size_t workspace_bytes, awa_stream_t stream)
{
    return forward_whole(plan, precision, heads, head_dim, in_dtype, video_qkv, video_token_stride, video_qkv_stride,
                         text_qkv, text_token_stride, text_qkv_stride, out_dtype, video_out, video_token_stride_out,
                         text_out, text_token_stride_out, workspace, workspace_bytes, stream, 1);
}

int awa_forward_prerotated(const awa_plan* plan, int precision, int heads, int head_dim, int in_dtype,
                           const void* video_qkv, int64_t video_token_stride, int64_t video_qkv_stride,
                           const void* text_qkv, int64_t text_token_stride, int64_t text_qkv_stride, int out_dtype,
                           void* video_out, int64_t video_token_stride_out, void* text_out,
                           int64_t text_token_stride_out, void* workspace, size_t workspace_bytes, awa_stream_t stream)
{
    return forward_whole(plan, precision, heads, head_dim, in_dtype, video_qkv, video_token_stride, video_qkv_stride,
                         text_qkv, text_token_stride, text_qkv_stride, out_dtype, video_out, video_token_stride_out,
                         text_out, text_token_stride_out, workspace, workspace_bytes, stream, 0);
}

static int forward_whole(const awa_plan* plan, int precision, int heads, int head_dim, int in_dtype,
                         const void* video_qkv, int64_t video_token_stride, int64_t video_qkv_stride,
                         const void* text_qkv, int64_t text_token_stride, int64_t text_qkv_stride, int out_dtype,
                         void* video_out, int64_t video_token_stride_out, void* text_out,
                         int64_t text_token_stride_out, void* workspace, size_t workspace_bytes, awa_stream_t stream,
                         int rotate)
{
    int rc = check_heads(plan, heads, head_dim);
    if (rc)
        return rc;
    if (!text_out || text_token_stride_out < (int64_t)heads * head_dim)
        return fail(AWA_ERR_INVALID, "awa_forward: invalid text output");
    int partial_dtype = AWA_F32;
    rc = forward_impl(plan, precision, heads, head_dim, 0, plan->info.window_count, in_dtype, video_qkv,
                      video_token_stride, video_qkv_stride, text_qkv, text_token_stride, text_qkv_stride, out_dtype,
                      video_out, video_token_stride_out, workspace, workspace_bytes, &partial_dtype, stream, rotate);
    if (rc)
        return rc;
    return launch_status(awa::launch_text_reduce(plan->dev, heads, head_dim, 0, partial_dtype, workspace,
                                                 (int64_t)heads * head_dim, 0, plan->info.window_count,
                                                 (float)plan->info.window_count, out_dtype, text_out,
                                                 text_token_stride_out, stream),
                         "awa_forward text reduce");
}

int awa_forward_windows(const awa_plan* plan, int precision, int heads, int head_dim, int window_begin,
                        int window_end, int in_dtype, const void* video_qkv, int64_t video_token_stride,
                        int64_t video_qkv_stride, const void* text_qkv, int64_t text_token_stride,
                        int64_t text_qkv_stride, int out_dtype, void* video_out, int64_t video_token_stride_out,
                        float* text_partial, void* workspace, size_t workspace_bytes, awa_stream_t stream)
{
    int rc = check_heads(plan, heads, head_dim);
    if (rc)
        return rc;
    if (window_begin < 0 || window_end > plan->info.window_count || window_begin > window_end || !text_partial)
        return fail(AWA_ERR_INVALID, "awa_forward_windows: invalid window range [%d, %d)", window_begin, window_end);
    if (window_begin == window_end)
        return launch_status(cudaMemsetAsync(text_partial, 0,
                                             (size_t)plan->info.text_tokens * heads * head_dim * sizeof(float), stream),
                             "memset text partial");
    int partial_dtype = AWA_F32;
    rc = forward_impl(plan, precision, heads, head_dim, window_begin, window_end, in_dtype, video_qkv,
                      video_token_stride, video_qkv_stride, text_qkv, text_token_stride, text_qkv_stride, out_dtype,
                      video_out, video_token_stride_out, workspace, workspace_bytes, &partial_dtype, stream);
    if (rc)
        return rc;
    // Unnormalised partial sum over this range, in window order.
    return launch_status(awa::launch_text_reduce(plan->dev, heads, head_dim, 0, partial_dtype, workspace,
                                                 (int64_t)heads * head_dim, window_begin, window_end, 0.f, AWA_F32,
                                                 text_partial, (int64_t)heads * head_dim, stream),
                         "awa_forward_windows text partial");
}

}  // extern "C"

namespace awa
{

int attention_range(const awa_plan* plan, int precision, int heads, int head_dim, int window_begin, int window_end,
                    int in_dtype, const void* video_qkv, int64_t video_token_stride, int64_t video_qkv_stride,
                    const void* text_qkv, int64_t text_token_stride, int64_t text_qkv_stride, int out_dtype,
                    void* video_out, int64_t video_token_stride_out, void* partials, size_t partial_bytes,
                    int* partial_dtype, cudaStream_t stream)
{
    int rc = check_heads(plan, heads, head_dim);
    if (rc)
        return rc;
    if (window_begin < 0 || window_end > plan->info.window_count || window_begin > window_end || !partial_dtype)
        return fail(AWA_ERR_INVALID, "attention range [%d, %d) invalid", window_begin, window_end);
    *partial_dtype = awa_attention_kernel_kind(plan, precision, in_dtype, heads, head_dim) == 1 ? AWA_BF16 : AWA_F32;
    if (window_begin == window_end)
        return AWA_OK;
    return forward_impl(plan, precision, heads, head_dim, window_begin, window_end, in_dtype, video_qkv,
                        video_token_stride, video_qkv_stride, text_qkv, text_token_stride, text_qkv_stride, out_dtype,
                        video_out, video_token_stride_out, partials, partial_bytes, partial_dtype, stream);
}

int attention_set(const awa_plan* plan, int precision, int heads, int head_dim, const int* windows, int count,
                  int in_dtype, const void* video_qkv, int64_t video_token_stride, int64_t video_qkv_stride,
                  const void* text_qkv, int64_t text_token_stride, int64_t text_qkv_stride, int out_dtype,
                  void* video_out, int64_t video_token_stride_out, void* partials, size_t partial_bytes,
                  int* partial_dtype, cudaStream_t stream)
{
    int rc = check_heads(plan, heads, head_dim);
    if (rc)
        return rc;
    if (count < 0 || (count > 0 && !windows) || !partial_dtype)
        return fail(AWA_ERR_INVALID, "attention over a window set: invalid set");
    *partial_dtype = awa_attention_kernel_kind(plan, precision, in_dtype, heads, head_dim) == 1 ? AWA_BF16 : AWA_F32;
    if (count == 0)
        return AWA_OK;
    return forward_impl(plan, precision, heads, head_dim, 0, plan->info.window_count, in_dtype, video_qkv,
                        video_token_stride, video_qkv_stride, text_qkv, text_token_stride, text_qkv_stride, out_dtype,
                        video_out, video_token_stride_out, partials, partial_bytes, partial_dtype, stream, 1, windows,
                        count);
}

int text_partial_sum(const awa_plan* plan, int heads, int head_dim, int partial_dtype, const void* partials,
                     int window_begin, int window_end, float* sum, cudaStream_t stream)
{
    int rc = check_heads(plan, heads, head_dim);
    if (rc)
        return rc;
    if (window_begin == window_end)
        return launch_status(cudaMemsetAsync(sum, 0, (size_t)plan->info.text_tokens * heads * head_dim * sizeof(float),
                                             stream),
                             "memset text partial");
    return launch_status(awa::launch_text_reduce(plan->dev, heads, head_dim, 0, partial_dtype, partials,
                                                 (int64_t)heads * head_dim, window_begin, window_end, 0.f, AWA_F32,
                                                 sum, (int64_t)heads * head_dim, stream),
                         "text partial sum");
}

}  // namespace awa

extern "C" {

int awa_text_finalize(const awa_plan* plan, int heads, int head_dim, const float* text_sum, int out_dtype,
                      void* text_out, int64_t text_token_stride, awa_stream_t stream)
{
    int rc = check_heads(plan, heads, head_dim);
    if (rc)
        return rc;
    if (!text_sum || !text_out || !valid_dtype(out_dtype) || text_token_stride < (int64_t)heads * head_dim)
        return fail(AWA_ERR_INVALID, "awa_text_finalize: invalid arguments");
    return launch_status(awa::launch_text_scale(plan->info.text_tokens, heads, head_dim, text_sum,
                                                (float)plan->info.window_count, out_dtype, text_out, text_token_stride,
                                                stream),
                         "awa_text_finalize");
}

int awa_qkv_project(int tokens, int model_dim, int heads, int head_dim, const void* x, int64_t x_stride,
                    const void* w, int64_t w_stride, const float* gamma_q, const float* gamma_k, float eps,
                    int out_dtype, void* out, int64_t out_stride, awa_stream_t stream)
{
    if (head_dim != 128)
        return fail(AWA_ERR_INVALID, "awa_qkv_project: head_dim %d (the tensor-core kernel needs 128)", head_dim);
    const int64_t n_out = 3 * (int64_t)heads * head_dim;
    if (tokens <= 0 || model_dim <= 0 || heads <= 0 || n_out > 0x7fffffff || !x || !w || !gamma_q || !gamma_k ||
        !out || !valid_dtype(out_dtype) || x_stride < model_dim || w_stride < model_dim || out_stride < n_out ||
        !(eps >= 0.f))
        return fail(AWA_ERR_INVALID, "awa_qkv_project: invalid sizes, dtype, eps or NULL tensor");
    const size_t osz = dtype_size(out_dtype);
    if (!is_aligned16(x) || !is_aligned16(w) || (x_stride * 2) % 16 || (w_stride * 2) % 16 ||
        reinterpret_cast<uintptr_t>(out) % 32 || (out_stride * (int64_t)osz) % 32)
        return fail(AWA_ERR_INVALID, "awa_qkv_project: x and w need 16-byte aligned rows, out 32-byte aligned rows");
    return launch_status(awa::launch_qkv_project(tokens, model_dim, heads, x, x_stride, w, w_stride, gamma_q, gamma_k,
                                                 eps, out_dtype, out, out_stride, static_cast<cudaStream_t>(stream)),
                         "awa_qkv_project launch");
}

int awa_qkv_project_rotated(int tokens, int model_dim, int heads, int head_dim, const void* x, int64_t x_stride,
                            const void* w, int64_t w_stride, const float* gamma_q, const float* gamma_k, float eps,
                            const awa_plan* plan, int branch, int out_dtype, void* out, int64_t out_stride,
                            awa_stream_t stream)
{
    int rc = check_heads(plan, heads, head_dim);
    if (rc)
        return rc;
    if (branch != AWA_BRANCH_VIDEO && branch != AWA_BRANCH_TEXT)
        return fail(AWA_ERR_INVALID, "awa_qkv_project_rotated: branch must be AWA_BRANCH_VIDEO or AWA_BRANCH_TEXT");
    const int rows = branch == AWA_BRANCH_VIDEO ? plan->info.source_tokens : plan->info.text_tokens;
    if (tokens != rows)
        return fail(AWA_ERR_INVALID, "awa_qkv_project_rotated: %d tokens, the plan's %s branch has %d", tokens,
                    branch == AWA_BRANCH_VIDEO ? "video" : "text", rows);
    if (head_dim < plan->info.rope_dim)
        return fail(AWA_ERR_INVALID, "awa_qkv_project_rotated: head_dim %d < rope_dim %d", head_dim,
                    plan->info.rope_dim);
    if (head_dim != 128)
        return fail(AWA_ERR_INVALID, "awa_qkv_project_rotated: head_dim %d (the tensor-core kernel needs 128)",
                    head_dim);
    const int64_t n_out = 3 * (int64_t)heads * head_dim;
    if (model_dim <= 0 || n_out > 0x7fffffff || !x || !w || !gamma_q || !gamma_k || !out || !valid_dtype(out_dtype) ||
        x_stride < model_dim || w_stride < model_dim || out_stride < n_out || !(eps >= 0.f))
        return fail(AWA_ERR_INVALID, "awa_qkv_project_rotated: invalid sizes, dtype, eps or NULL tensor");
    const size_t osz = dtype_size(out_dtype);
    if (!is_aligned16(x) || !is_aligned16(w) || (x_stride * 2) % 16 || (w_stride * 2) % 16 ||
        reinterpret_cast<uintptr_t>(out) % 32 || (out_stride * (int64_t)osz) % 32)
        return fail(AWA_ERR_INVALID,
                    "awa_qkv_project_rotated: x and w need 16-byte aligned rows, out 32-byte aligned rows");
    return launch_status(awa::launch_qkv_project(tokens, model_dim, heads, x, x_stride, w, w_stride, gamma_q, gamma_k,
                                                 eps, out_dtype, out, out_stride, static_cast<cudaStream_t>(stream),
                                                 &plan->dev, branch == AWA_BRANCH_VIDEO ? 1 : 2),
                         "awa_qkv_project_rotated launch");
}

int awa_out_project(int tokens, int in_dim, int out_dim, const void* x, int64_t x_stride, const void* w,
                    int64_t w_stride, const float* bias, const float* gate, const void* residual,
                    int64_t residual_stride, int residual_dtype, int out_dtype, void* out, int64_t out_stride,
                    awa_stream_t stream)
{
    if (tokens <= 0 || in_dim <= 0 || out_dim <= 0 || out_dim % 128 || !x || !w || !bias || !gate || !residual ||
        !out || !valid_dtype(out_dtype) || !valid_dtype(residual_dtype) || x_stride < in_dim ||
        w_stride < in_dim || out_stride < out_dim || residual_stride < out_dim)
        return fail(AWA_ERR_INVALID, "awa_out_project: invalid sizes (out_dim a multiple of 128), dtype or NULL");
    const size_t osz = dtype_size(out_dtype), rsz = dtype_size(residual_dtype);
    if (!is_aligned16(x) || !is_aligned16(w) || !is_aligned16(residual) || (x_stride * 2) % 16 ||
        (w_stride * 2) % 16 || (residual_stride * (int64_t)rsz) % 16 || reinterpret_cast<uintptr_t>(out) % 32 ||
        (out_stride * (int64_t)osz) % 32)
        return fail(AWA_ERR_INVALID,
                    "awa_out_project: x, w, residual need 16-byte aligned rows, out 32-byte aligned rows");
    return launch_status(awa::launch_out_project(tokens, in_dim, out_dim, x, x_stride, w, w_stride, bias, gate,
                                                 residual, residual_stride, residual_dtype, out_dtype, out,
                                                 out_stride, static_cast<cudaStream_t>(stream)),
                         "awa_out_project launch");
}

int64_t awa_window_range_video_rows(const awa_plan* plan, int window_begin, int window_end)
{
    if (!plan || window_begin < 0 || window_end > plan->info.window_count || window_begin > window_end)
        return -1;
    int64_t rows = 0;
    for (int w = window_begin; w < window_end; w++)
        rows += plan->descs[w].video;
    return rows;
}

static int shard_copy(const awa_plan* plan, int heads, int head_dim, int window_begin, int window_end, int dtype,
                      const void* src, int64_t src_stride, void* dst, int64_t dst_stride, int to_source,
                      cudaStream_t stream)
{
    int rc = check_heads(plan, heads, head_dim);
    if (rc)
        return rc;
    if (window_begin < 0 || window_end > plan->info.window_count || window_begin > window_end || !src || !dst ||
        !valid_dtype(dtype))
        return fail(AWA_ERR_INVALID, "shard copy: invalid arguments");
    if (window_begin == window_end)
        return AWA_OK;
    return launch_status(awa::launch_shard_copy(plan->dev, heads, head_dim, window_begin, window_end, dtype, src,
                                                src_stride, dst, dst_stride, to_source, stream),
                         "shard copy");
}

int awa_scatter_video_shard(const awa_plan* plan, int heads, int head_dim, int window_begin, int window_end,
                            int dtype, const void* shard, void* video_out, int64_t video_token_stride,
                            awa_stream_t stream)
{
    return shard_copy(plan, heads, head_dim, window_begin, window_end, dtype, shard, (int64_t)heads * head_dim,
                      video_out, video_token_stride, 1, stream);
}

int awa_gather_video_shard(const awa_plan* plan, int heads, int head_dim, int window_begin, int window_end,
                           int dtype, const void* video, int64_t video_token_stride, void* shard,
                           awa_stream_t stream)
{
    return shard_copy(plan, heads, head_dim, window_begin, window_end, dtype, video, video_token_stride, shard,
                      (int64_t)heads * head_dim, 0, stream);
}

int awa_partition_windows(const awa_plan* plan, int parts, int* bounds)
{
    if (!plan || parts <= 0 || !bounds)
        return fail(AWA_ERR_INVALID, "awa_partition_windows: invalid arguments");
    const int W = plan->info.window_count;
    double total = 0;
    for (double c : plan->window_cost)
        total += c;
    bounds[0] = 0;
    double acc = 0;
    int w = 0;
    for (int p = 1; p < parts; p++)
    {
        const double target = total * p / parts;
        while (w < W && acc + plan->window_cost[w] * 0.5 < target)
            acc += plan->window_cost[w++];
        bounds[p] = std::max(w, bounds[p - 1]);
    }
    bounds[parts] = W;
    return AWA_OK;
}

int awa_selftest_bounded_wait(unsigned limit_us, int* observed, awa_stream_t stream)
{
    if (limit_us == 0 || limit_us > 1000000u || !observed)
        return fail(AWA_ERR_INVALID, "awa_selftest_bounded_wait: limit must be 1..1000000 us");
    int* flag = awa::device_error_flag();
    if (!flag)
        return fail(AWA_ERR_CUDA, "device status flag unavailable");
    int* d_observed = nullptr;
    cudaError_t err = cudaMalloc(&d_observed, sizeof(int));
    if (err != cudaSuccess)
        return cuda_fail(err, "self-test buffer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    err = cudaMemsetAsync(d_observed, 0, sizeof(int), s);
    if (err == cudaSuccess)
        err = static_cast<cudaError_t>(awa::launch_wait_selftest((uint64_t)limit_us * 1000ull, flag, d_observed, s));
    if (err == cudaSuccess)
        err = cudaMemcpyAsync(observed, d_observed, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess)
        err = cudaStreamSynchronize(s);
    cudaFree(d_observed);
    return err == cudaSuccess ? AWA_OK : cuda_fail(err, "awa_selftest_bounded_wait");
}

int awa_device_status(void)
{
    int* flag = awa::device_error_flag();
    if (!flag)
        return fail(AWA_ERR_CUDA, "device status flag unavailable");
    cudaError_t err = cudaDeviceSynchronize();
    if (err != cudaSuccess)
        return cuda_fail(err, "cudaDeviceSynchronize");
    int value = 0;
    err = cudaMemcpy(&value, flag, sizeof(int), cudaMemcpyDeviceToHost);
    if (err != cudaSuccess)
        return cuda_fail(err, "read device status");
    if (value != 0)
    {
        cudaMemset(flag, 0, sizeof(int));
        return fail(AWA_ERR_DEVICE, "device check failed with code %d", value);
    }
    return AWA_OK;
}

}  // extern "C"
