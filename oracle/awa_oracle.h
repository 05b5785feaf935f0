/*
 * awa_oracle.h -- CPU restatement of SeedVR2-ncnn's adaptive window attention
 * (AWA) layer chain, used ONLY as the parity checker of the CUDA path.
 *
 * TEST INFRASTRUCTURE. Nothing in the product (seedvr2-ncnn_b200/, include/)
 * links or calls this code; only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py do.
 *
 * Every function restates one reference function of
 * src/awa/awa_layers.cpp (HGinkgo/SeedVR2-ncnn) in plain C, with the same
 * loop order and the same fp32 operation order, so that integer outputs
 * (windows, index maps) and copy outputs (pack, unpack video rows) are
 * bit-identical to the reference, and the fp32 arithmetic (RoPE rotation,
 * text mean) is bit-identical when the inputs are.
 *
 * Pinning: the restatement is checked against (a) the reference's own
 * awa_layers.cpp compiled here unmodified (oracle/_ref, see Makefile) and
 * (b) golden vectors written by the reference's PyTorch mirror
 * (tools/reference/awa_attention.py, seedvr2_baseline.py, dit_block.py),
 * stored in tests/golden/ with the script that made them.
 *
 * Layouts (dense, row-major, fp32):
 *   video QKV  [N_v][3][H][d]     (token, q/k/v, head, feature)
 *   text QKV   [T_txt][3][H][d]
 *   packed QKV [S][3][H][d]       S = sum over windows of (video tokens + T_txt)
 *   attended   [S][H][d]
 *   video out  [N_v][H][d], text out [T_txt][H][d]
 */
#ifndef AWA_ORACLE_H
#define AWA_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Window bounds [t0,t1) x [h0,h1) x [w0,w1); out6 holds 6 ints per window. */
int oracle_make_windows(int source_t, int source_h, int source_w, int num_t, int num_h, int num_w,
                        int shifted, int* out6, int capacity);

/* Index maps of one layer configuration (awa_layers.cpp:382-407, 599-626).
 * sequence_index[S], cu_seqlens[W+1], video_positions[N_v], text_positions[W*T_txt].
 * Returns S (packed sequence length) or -1. Any output pointer may be NULL. */
int oracle_index_maps(int source_t, int source_h, int source_w, int num_t, int num_h, int num_w,
                      int text_tokens, int shifted, int* sequence_index, int* cu_seqlens,
                      int* video_positions, int* text_positions);

/* Pack (awa_layers.cpp:419-458): packed[pos] = (video|text)[sequence_index[pos]]. */
void oracle_pack(const float* video_qkv, const float* text_qkv, int source_tokens, int heads, int head_dim,
                 const int* sequence_index, int sequence_tokens, float* packed);

/* MMRoPE table (awa_layers.cpp:867-911): rotations[S][2*rope_dim]. */
int oracle_rope_table(int source_t, int source_h, int source_w, int num_t, int num_h, int num_w,
                      int text_tokens, int shifted, int rope_dim, float* rotations);

/* MMRoPE forward (awa_layers.cpp:913-953). */
void oracle_rope(const float* packed_in, int sequence_tokens, int heads, int head_dim, int rope_dim,
                 const float* rotations, float* packed_out);

/* WindowAttention forward (awa_layers.cpp:1062-1120). window_offsets = cu_seqlens.
 * num_threads > 1 splits (window, head) pairs over OpenMP threads; every output
 * element is computed by one thread with the reference's sequential order, so
 * the result does not depend on the thread count. */
void oracle_attention(const float* packed, int window_count, const int* window_offsets, int heads,
                      int head_dim, float* attended, int num_threads);

/* Same, restricted to windows [first, last) (for bounded CPU timing samples). */
void oracle_attention_range(const float* packed, int first_window, int last_window, const int* window_offsets,
                            int heads, int head_dim, float* attended, int num_threads);

/* Unpack forward (awa_layers.cpp:638-689), non-batched video layout. */
int oracle_unpack(const float* attended, int sequence_tokens, int source_tokens, int heads, int head_dim,
                  int window_count, int text_tokens, const int* video_positions, const int* text_positions,
                  float* video_out, float* text_out);

/* Round-to-nearest-even fp32 -> bf16 -> fp32 (for bf16 test inputs). */
void oracle_round_bf16(const float* in, float* out, int64_t count);

#ifdef __cplusplus
}
#endif

#endif
