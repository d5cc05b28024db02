/*
 * mt_graph.h — host-side graph substitution engine (libmt_graph.so).
 *
 * The native half of certified graph substitution: find every occurrence of
 * a region's original-op pattern in a traced model graph, order the graph
 * with the accepted occurrences replaced by one region node each, and prove
 * that two graphs compute the same thing (same operations, same leaves, same
 * sharing). It replaces the reference's MLX-graph extension
 * autotuner_runtime/graph_native/graph_native.cpp (match :38-86, rewrite
 * :108-259, same_structure :261-290, same_computation :292-322) and its
 * Python entry points autotuner_runtime/graph_native/__init__.py:127-141.
 *
 * Graphs are flat node tables in topological order (every input index is
 * smaller than the node's own). A node is either a leaf (op == 0; `leaf`
 * names its value: two leaves with equal `leaf` are the same value) or an
 * operation (op != 0; `op` is the caller's interned key of the operation
 * and its non-tensor attributes, so equal keys mean the same computation on
 * equal inputs). Every node also carries `type`, the interned shape and
 * dtype of its value, compared wherever two nodes are paired (parameters
 * included). The caller (Python, from a torch.fx
 * graph) builds the keys; the engine only compares them. No CUDA, no
 * allocation visible to the caller, thread-compatible (no global state).
 *
 * Every function returns >= 0 on success and a negative MT_GRAPH_ERR_* code
 * on failure; mt_graph_error_string() describes the last failure of the
 * calling thread.
 */
#ifndef MT_GRAPH_H
#define MT_GRAPH_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MT_GRAPH_ERR_ARG (-1)        /* malformed table or argument */
#define MT_GRAPH_ERR_CAPACITY (-2)   /* an output buffer is too small */
#define MT_GRAPH_ERR_UNUSED (-3)     /* a pattern parameter is not reached from its outputs */
#define MT_GRAPH_ERR_CYCLE (-4)      /* a replacement would make the graph cyclic */

typedef struct mt_graph_view {
  int32_t n_nodes;
  const int64_t* op;      /* [n_nodes] interned operation key; 0 for a leaf */
  const int64_t* type;    /* [n_nodes] interned shape and dtype of the node's value; equal for every bound pair */
  const int64_t* leaf;    /* [n_nodes] identity of a leaf's value (read where op == 0) */
  const int32_t* in_off;  /* [n_nodes + 1] offsets into in_idx */
  const int32_t* in_idx;  /* the inputs of node i: in_idx[in_off[i] .. in_off[i+1]) */
} mt_graph_view;

/* Occurrences of a pattern in a graph (reference graph_native.cpp:108-178).
 *
 * The pattern's boundary is its free parameters `params` (leaf nodes of the
 * pattern that bind to any graph node of the same position in the
 * computation; two parameters may bind the same node, as in x + x) and its
 * outputs `outs` (operation nodes). Every other pattern leaf must meet a
 * graph leaf of the same identity. Non-parameter pattern nodes bind distinct
 * graph nodes, outputs of one occurrence are never outputs of another, and
 * an occurrence whose bound inputs are computed inside it is skipped.
 * anchors[i] >= 0 fixes parameter i to that graph node before matching
 * (NULL: none fixed). The search starts from the last output, in graph
 * order, so occurrences are found in the order they compute.
 *
 * occ receives, per occurrence, n_params bound graph nodes (in the order of
 * `params`) then n_outs bound graph nodes (in the order of `outs`); at most
 * max_occ occurrences are written. Returns the number found (which may
 * exceed max_occ: call again with room), or a negative error. */
int mt_graph_find(const mt_graph_view* graph, const mt_graph_view* pattern, const int32_t* params,
                  int32_t n_params, const int32_t* outs, int32_t n_outs, const int32_t* anchors,
                  int32_t* occ, int32_t max_occ);

/* The rewritten graph's node order (reference graph_native.cpp:180-259).
 *
 * occ holds n_occ occurrences laid out as mt_graph_find writes them;
 * accept[k] != 0 replaces occurrence k by one region node whose inputs are
 * its bound parameters and whose outputs stand for its bound outputs
 * everywhere they are used; a declined occurrence keeps its original nodes.
 * The nodes the roots need (after the replacement) are listed in a valid
 * order: order[2*i] is 0 for an original node (order[2*i+1] its index in
 * the graph) or 1 for a region node (order[2*i+1] the occurrence). Nodes no
 * root needs any more are left out. Returns the number of entries (at most
 * cap), MT_GRAPH_ERR_CAPACITY when cap is too small, or MT_GRAPH_ERR_CYCLE
 * when a region's inputs depend on its own outputs. */
int mt_graph_order(const mt_graph_view* graph, const int32_t* roots, int32_t n_roots, const int32_t* occ,
                   int32_t n_occ, int32_t n_params, int32_t n_outs, const uint8_t* accept, int32_t* order,
                   int32_t cap);

/* Structural equality of two graphs from their roots (reference
 * graph_native.cpp:261-322): a one-to-one correspondence of the nodes the
 * roots reach, with equal operation keys, equal leaf identities, inputs in
 * the same order, and the same sharing (a node used twice on one side is one
 * node used twice on the other). Callers choose what a leaf identity means:
 * the tensor object (same_structure) or its bytes (same_computation).
 * Returns 1 when equal, 0 when not (reason written, NUL-terminated, into
 * reason[0 .. reason_len)), or a negative error. */
int mt_graph_same(const mt_graph_view* a, const int32_t* roots_a, const mt_graph_view* b, const int32_t* roots_b,
                  int32_t n_roots, char* reason, int32_t reason_len);

/* Description of the calling thread's last failure ("" if none). */
const char* mt_graph_error_string(void);

/* Version of the engine's table format: bumped when a layout above changes. */
int mt_graph_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MT_GRAPH_H */
