/*
 * awa_package.h -- model-package side of the B200 AWA library: reading the
 * AWA layer lines of an ncnn block graph (.param text), writing its
 * resolution-independent form (the -1 grid sentinel), and checking a model
 * package against its manifest.sha256. Host only; no CUDA call, no device.
 * Status codes and awa_last_error() as in awa_b200.h.
 *
 * These let a package exported for the reference's ncnn layers run on the
 * B200 layers unchanged: the chain's ParamDict values come out of the graph
 * as an awa_layer_params, and awa_plan_create(&chain.params, &spec, ...) with
 * the session's runtime spec replaces the four layers' load_param.
 */
#ifndef AWA_PACKAGE_H
#define AWA_PACKAGE_H

#include <stddef.h>

#include "awa_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* One Pack -> MMRoPE -> WindowAttention -> Unpack chain of an ncnn graph, as
 * the exporter writes it (tools/export_dit_block.py:578-644 of the reference):
 *   SeedVR2AWAPack          <name> 2 2 <video> <text> <packed> <cu_seqlens> 0=.. 7=..
 *   SeedVR2MMRoPE           <name> 1 1 <packed> <roped> 0=.. 7=.. 8=126
 *   SeedVR2WindowAttention  <name> 1 1 <roped> <attended> 0=.. 7=..
 *   SeedVR2AWAUnpack        <name> 1 2 <attended> <video> <text> 0=.. 7=..
 *   Reshape reshape_awa_video_batch 1 1 <video> <batch> 0=2560 1=<N_v or -1>
 * MMRoPE and WindowAttention may be absent (a graph that kept those steps as
 * ordinary ncnn layers); the chain then links Pack and Unpack only. */
typedef struct
{
    awa_layer_params params; /* ParamDict 0-8 of the chain (identical on its layers); rope_dim is
                                MMRoPE's id 8 (126 when absent, as pd.get(8, 126)) */
    int dynamic;             /* 1: source_t/h/w are -1,-1,-1, the grid comes from the runtime spec */
    int pack_line;           /* 1-based line numbers in the text; 0 = layer absent */
    int rope_line;
    int attention_line;
    int unpack_line;
    int reshape_line;        /* the Reshape fed by Unpack's video output; 0 = none */
    int reshape_height;      /* its parameter 1: N_v (static) or -1 (dynamic); 0 when absent */
} awa_graph_chain;

/* Reads an ncnn .param text (magic 7767517, "<layers> <blobs>", one layer per
 * line: type name bottoms tops blob-names id=value ...) and returns the number
 * of AWA chains in it, filling min(count, capacity) entries of chains in Pack
 * order. Checks what ncnn's loader and the AWA layers' load_param would reject
 * (header, layer count, blob declarations; on AWA lines integer id=value
 * pairs with no id repeated, the load_common grid rule awa_layers.cpp:90-114:
 * ids 0-2 all -1 or all positive, ids 3-6 positive, id 7 defaulting to 0;
 * rope_dim a positive multiple of 6, :872-874), that ids 0-7 are equal along a
 * chain, the blob arity of each layer, and the chain's wiring (each AWA layer
 * consumes its AWA predecessor's first output; the k-th Pack pairs with the
 * k-th Unpack). Returns
 * -1 with awa_last_error() set when the graph is malformed; 0 when it holds no
 * AWA layer. */
int awa_graph_find_chains(const char* param_text, size_t length, awa_graph_chain* chains, int capacity);
int awa_graph_find_chains_file(const char* param_path, awa_graph_chain* chains, int capacity);

/* Replaces normalize_dynamic_awa_template (tools/export_dit_block.py:38-124):
 * rewrites ids 0, 1, 2 of every AWA line to -1 and the height (id 1) of the
 * Reshape "reshape_awa_video_batch" fed by the Unpack video output to -1,
 * leaving every other line as it was, with the same checks and the same bytes
 * out (lines joined by '\n', one trailing '\n'). Writes the result into out
 * (capacity bytes, NUL-terminated when it fits) and its length to *out_length;
 * returns 0, -1 for a graph the reference function rejects, or -100 when
 * capacity is too small (*out_length then holds the size needed, without the
 * NUL). */
int awa_graph_make_dynamic(const char* param_text, size_t length, char* out, size_t capacity,
                           size_t* out_length);

/* Replaces validate_manifest (src/model/model_registry.cpp:248-362): the
 * package directory's manifest.sha256 lists "<64 hex>  <relative path>" per
 * line (CR LF accepted, blank lines skipped, hex case-insensitive); every path
 * is relative without "." or ".." components or backslashes, listed once; the
 * package holds no symbolic link; every listed file exists with that SHA-256
 * and every regular file but the manifest is listed. expected_records: 0 = the
 * reference's package rule (75 records, or 146 with CFG), > 0 = exactly that
 * many, < 0 = any number. Returns 0, or -1 with the reference's message in
 * awa_last_error(). */
int awa_manifest_validate(const char* package_dir, int expected_records);

/* SHA-256 (FIPS 180-4) as 64 lowercase hex digits plus NUL into hex[65]. */
int awa_sha256(const void* data, size_t size, char* hex);
int awa_sha256_file(const char* path, char* hex);

#ifdef __cplusplus
}
#endif

#endif /* AWA_PACKAGE_H */
