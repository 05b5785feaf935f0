/*
 * awa_oracle.c -- CPU restatement of the SeedVR2-ncnn AWA layer chain.
 * TEST INFRASTRUCTURE ONLY (parity checker); see awa_oracle.h.
 *
 * Compile with -ffp-contract=off: the reference is built for baseline x86-64
 * (no FMA), so each fp32 multiply and add rounds separately there too.
 */
#include "awa_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* awa_layers.cpp:36-39 */
static int ceil_div_int(int numerator, int denominator)
{
    return (numerator + denominator - 1) / denominator;
}

/* awa_layers.cpp:41-51: Python's round() (half to even) for non-negative values. */
static int round_half_even_positive(double value)
{
    const double lower = floor(value);
    const double fraction = value - lower;
    if (fraction < 0.5)
        return (int)lower;
    if (fraction > 0.5)
        return (int)(lower + 1.0);
    {
        const int lower_int = (int)lower;
        return lower_int % 2 == 0 ? lower_int : lower_int + 1;
    }
}

/* awa_layers.cpp:53-88 (mirror of tools/reference/seedvr2_baseline.py:37-79).
 * Area-normalised window size against a 45x80 grid, optional half-window
 * shift per axis, clipped bounds, loop order w (outer), h, t (inner). */
int oracle_make_windows(int source_t, int source_h, int source_w, int num_t, int num_h, int num_w,
                        int shifted, int* out6, int capacity)
{
    if (source_t <= 0 || source_h <= 0 || source_w <= 0 || num_t <= 0 || num_h <= 0 || num_w <= 0)
        return 0;
    const double scale = sqrt(3600.0 / (source_h * source_w));
    const int resized_h = round_half_even_positive(source_h * scale);
    const int resized_w = round_half_even_positive(source_w * scale);
    const int window_h = ceil_div_int(resized_h, num_h);
    const int window_w = ceil_div_int(resized_w, num_w);
    const int window_t = ceil_div_int(source_t < 30 ? source_t : 30, num_t);
    const double shift_t = shifted && window_t < source_t ? 0.5 : 0.0;
    const double shift_h = shifted && window_h < source_h ? 0.5 : 0.0;
    const double shift_w = shifted && window_w < source_w ? 0.5 : 0.0;
    const int count_t = (int)ceil((source_t - shift_t) / window_t) + (shift_t > 0 ? 1 : 0);
    const int count_h = (int)ceil((source_h - shift_h) / window_h) + (shift_h > 0 ? 1 : 0);
    const int count_w = (int)ceil((source_w - shift_w) / window_w) + (shift_w > 0 ? 1 : 0);
    int count = 0;
    for (int iw = 0; iw < count_w; iw++)
        for (int ih = 0; ih < count_h; ih++)
            for (int it = 0; it < count_t; it++)
            {
                int t0 = (int)((it - shift_t) * window_t);
                int h0 = (int)((ih - shift_h) * window_h);
                int w0 = (int)((iw - shift_w) * window_w);
                int t1 = (int)((it - shift_t + 1.0) * window_t);
                int h1 = (int)((ih - shift_h + 1.0) * window_h);
                int w1 = (int)((iw - shift_w + 1.0) * window_w);
                t0 = t0 > 0 ? t0 : 0;
                h0 = h0 > 0 ? h0 : 0;
                w0 = w0 > 0 ? w0 : 0;
                t1 = t1 < source_t ? t1 : source_t;
                h1 = h1 < source_h ? h1 : source_h;
                w1 = w1 < source_w ? w1 : source_w;
                if (t1 > t0 && h1 > h0 && w1 > w0)
                {
                    if (out6 && count < capacity)
                    {
                        int* o = out6 + 6 * count;
                        o[0] = t0; o[1] = t1; o[2] = h0; o[3] = h1; o[4] = w0; o[5] = w1;
                    }
                    count++;
                }
            }
    return count;
}

static int* windows_alloc(int source_t, int source_h, int source_w, int num_t, int num_h, int num_w, int shifted,
                          int* count)
{
    const int n = oracle_make_windows(source_t, source_h, source_w, num_t, num_h, num_w, shifted, NULL, 0);
    int* windows = (int*)malloc(sizeof(int) * 6 * (size_t)(n > 0 ? n : 1));
    oracle_make_windows(source_t, source_h, source_w, num_t, num_h, num_w, shifted, windows, n);
    *count = n;
    return windows;
}

/* Pack::load_param (awa_layers.cpp:382-407) and Unpack::load_param (599-626):
 * window video tokens in (t, h, w) row-major order, then the text tokens,
 * for every window in make_windows order. */
int oracle_index_maps(int source_t, int source_h, int source_w, int num_t, int num_h, int num_w,
                      int text_tokens, int shifted, int* sequence_index, int* cu_seqlens,
                      int* video_positions, int* text_positions)
{
    int count = 0;
    int* windows = windows_alloc(source_t, source_h, source_w, num_t, num_h, num_w, shifted, &count);
    const int source_tokens = source_t * source_h * source_w;
    if (video_positions)
        for (int i = 0; i < source_tokens; i++)
            video_positions[i] = -1;
    int cursor = 0;
    if (cu_seqlens)
        cu_seqlens[0] = 0;
    for (int wi = 0; wi < count; wi++)
    {
        const int* win = windows + 6 * wi;
        for (int t = win[0]; t < win[1]; t++)
            for (int h = win[2]; h < win[3]; h++)
                for (int w = win[4]; w < win[5]; w++)
                {
                    const int source_index = (t * source_h + h) * source_w + w;
                    if (sequence_index)
                        sequence_index[cursor] = source_index;
                    if (video_positions)
                        video_positions[source_index] = cursor;
                    cursor++;
                }
        for (int token = 0; token < text_tokens; token++)
        {
            if (sequence_index)
                sequence_index[cursor + token] = source_tokens + token;
            if (text_positions)
                text_positions[wi * text_tokens + token] = cursor + token;
        }
        cursor += text_tokens;
        if (cu_seqlens)
            cu_seqlens[wi + 1] = cursor;
    }
    free(windows);
    return count > 0 ? cursor : -1;
}

/* awa_layers.cpp:440-454 */
void oracle_pack(const float* video_qkv, const float* text_qkv, int source_tokens, int heads, int head_dim,
                 const int* sequence_index, int sequence_tokens, float* packed)
{
    const size_t row = (size_t)3 * heads * head_dim;
    for (int position = 0; position < sequence_tokens; position++)
    {
        const int source_index = sequence_index[position];
        const float* source = source_index < source_tokens
                                  ? video_qkv + (size_t)source_index * row
                                  : text_qkv + (size_t)(source_index - source_tokens) * row;
        memcpy(packed + (size_t)position * row, source, row * sizeof(float));
    }
}

/* awa_layers.cpp:876-910: per packed position, cos then sin of each rotated
 * feature; the frequency of pair p on an axis of axis_dim features is
 * powf(10000, -(2p)/axis_dim); video coordinates are window-local with the t
 * axis offset by the text count, text token i has coordinates (i, i, i). */
static void write_rotation(float* data, int rope_dim, int ct, int ch, int cw)
{
    const int axis_dim = rope_dim / 3;
    const int coordinates[3] = {ct, ch, cw};
    for (int axis = 0; axis < 3; axis++)
        for (int pair = 0; pair < axis_dim / 2; pair++)
        {
            const float frequency = powf(10000.f, -(float)(2 * pair) / (float)axis_dim);
            const float angle = (float)coordinates[axis] * frequency;
            const int feature = axis * axis_dim + 2 * pair;
            data[feature] = cosf(angle);
            data[feature + 1] = data[feature];
            data[rope_dim + feature] = sinf(angle);
            data[rope_dim + feature + 1] = data[rope_dim + feature];
        }
}

int oracle_rope_table(int source_t, int source_h, int source_w, int num_t, int num_h, int num_w,
                      int text_tokens, int shifted, int rope_dim, float* rotations)
{
    if (rope_dim <= 0 || rope_dim % 6 != 0)
        return -1;
    int count = 0;
    int* windows = windows_alloc(source_t, source_h, source_w, num_t, num_h, num_w, shifted, &count);
    int cursor = 0;
    for (int wi = 0; wi < count; wi++)
    {
        const int* win = windows + 6 * wi;
        for (int t = win[0]; t < win[1]; t++)
            for (int h = win[2]; h < win[3]; h++)
                for (int w = win[4]; w < win[5]; w++)
                    write_rotation(rotations + (size_t)(cursor++) * 2 * rope_dim, rope_dim, text_tokens + (t - win[0]),
                                   h - win[2], w - win[4]);
        for (int token = 0; token < text_tokens; token++)
            write_rotation(rotations + (size_t)(cursor++) * 2 * rope_dim, rope_dim, token, token, token);
    }
    free(windows);
    return cursor;
}

/* awa_layers.cpp:930-951: Q and K rows (qkv_head < 2H), features < rope_dim,
 * interleaved pairs; V rows and the tail features are copied. */
void oracle_rope(const float* packed_in, int sequence_tokens, int heads, int head_dim, int rope_dim,
                 const float* rotations, float* packed_out)
{
    const int rows = 3 * heads;
    for (int token = 0; token < sequence_tokens; token++)
    {
        const float* source = packed_in + (size_t)token * rows * head_dim;
        float* output = packed_out + (size_t)token * rows * head_dim;
        const float* rotation = rotations + (size_t)token * 2 * rope_dim;
        for (int qkv_head = 0; qkv_head < rows; qkv_head++)
            for (int feature = 0; feature < head_dim; feature++)
            {
                const int offset = qkv_head * head_dim + feature;
                if (qkv_head >= 2 * heads || feature >= rope_dim)
                {
                    output[offset] = source[offset];
                    continue;
                }
                const int paired_feature = feature % 2 == 0 ? feature + 1 : feature - 1;
                const float paired = source[qkv_head * head_dim + paired_feature];
                const float a = source[offset] * rotation[feature];
                const float b = paired * rotation[rope_dim + feature];
                output[offset] = feature % 2 == 0 ? a - b : a + b;
            }
    }
}

/* awa_layers.cpp:1080-1117: per window, head and query, naive dot products,
 * max subtraction, expf, sequential normaliser, then out = sum_k (p/norm)*v. */
static void attention_window_head(const float* packed, int window_start, int window_length, int head, int heads,
                                  int head_dim, float* attended, float* scores)
{
    const float scale = 1.f / sqrtf((float)head_dim);
    const size_t in_row = (size_t)3 * heads * head_dim;
    const size_t out_row = (size_t)heads * head_dim;
    for (int query = 0; query < window_length; query++)
    {
        const float* query_data = packed + (size_t)(window_start + query) * in_row + (size_t)head * head_dim;
        float max_score = -INFINITY;
        for (int key = 0; key < window_length; key++)
        {
            const float* key_data = packed + (size_t)(window_start + key) * in_row + (size_t)(heads + head) * head_dim;
            float dot = 0.f;
            for (int feature = 0; feature < head_dim; feature++)
                dot += query_data[feature] * key_data[feature];
            scores[key] = dot * scale;
            max_score = max_score > scores[key] ? max_score : scores[key];
        }
        float normalizer = 0.f;
        for (int key = 0; key < window_length; key++)
        {
            scores[key] = expf(scores[key] - max_score);
            normalizer += scores[key];
        }
        float* output = attended + (size_t)(window_start + query) * out_row + (size_t)head * head_dim;
        for (int feature = 0; feature < head_dim; feature++)
        {
            float value = 0.f;
            for (int key = 0; key < window_length; key++)
            {
                const float* value_data =
                    packed + (size_t)(window_start + key) * in_row + (size_t)(2 * heads + head) * head_dim;
                value += scores[key] / normalizer * value_data[feature];
            }
            output[feature] = value;
        }
    }
}

void oracle_attention_range(const float* packed, int first_window, int last_window, const int* window_offsets,
                            int heads, int head_dim, float* attended, int num_threads)
{
    const int pairs = (last_window - first_window) * heads;
    int max_length = 1;
    for (int w = first_window; w < last_window; w++)
    {
        const int length = window_offsets[w + 1] - window_offsets[w];
        max_length = length > max_length ? length : max_length;
    }
#ifdef _OPENMP
    if (num_threads < 1)
        num_threads = 1;
#pragma omp parallel num_threads(num_threads)
#endif
    {
        float* scores = (float*)malloc(sizeof(float) * (size_t)max_length);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int pair = 0; pair < pairs; pair++)
        {
            const int window = first_window + pair / heads;
            const int head = pair % heads;
            const int start = window_offsets[window];
            attention_window_head(packed, start, window_offsets[window + 1] - start, head, heads, head_dim, attended,
                                  scores);
        }
        free(scores);
    }
    (void)num_threads;
}

void oracle_attention(const float* packed, int window_count, const int* window_offsets, int heads, int head_dim,
                      float* attended, int num_threads)
{
    oracle_attention_range(packed, 0, window_count, window_offsets, heads, head_dim, attended, num_threads);
}

/* awa_layers.cpp:659-687: video rows copied back by video_positions; text
 * rows accumulate x / W over windows in window order. */
int oracle_unpack(const float* attended, int sequence_tokens, int source_tokens, int heads, int head_dim,
                  int window_count, int text_tokens, const int* video_positions, const int* text_positions,
                  float* video_out, float* text_out)
{
    const size_t row = (size_t)heads * head_dim;
    for (int source_index = 0; source_index < source_tokens; source_index++)
    {
        const int packed_index = video_positions[source_index];
        if (packed_index < 0 || packed_index >= sequence_tokens)
            return -1;
        memcpy(video_out + (size_t)source_index * row, attended + (size_t)packed_index * row, row * sizeof(float));
    }
    memset(text_out, 0, sizeof(float) * row * (size_t)text_tokens);
    for (int window = 0; window < window_count; window++)
        for (int token = 0; token < text_tokens; token++)
        {
            const float* packed_data = attended + (size_t)text_positions[window * text_tokens + token] * row;
            float* text_data = text_out + (size_t)token * row;
            for (size_t value = 0; value < row; value++)
                text_data[value] += packed_data[value] / (float)window_count;
        }
    return 0;
}

void oracle_round_bf16(const float* in, float* out, int64_t count)
{
    for (int64_t i = 0; i < count; i++)
    {
        uint32_t bits;
        memcpy(&bits, in + i, 4);
        if ((bits & 0x7f800000u) == 0x7f800000u && (bits & 0x007fffffu))
            bits |= 0x00400000u; /* quiet NaN stays NaN */
        else
            bits = (bits + 0x7fffu + ((bits >> 16) & 1u)) & 0xffff0000u;
        memcpy(out + i, &bits, 4);
    }
}
