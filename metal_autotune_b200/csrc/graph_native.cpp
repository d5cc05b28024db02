// Host-side graph substitution engine behind include/mt_graph.h.
//
// The reference rewrites MLX's lazy array graph in C++
// (autotuner_runtime/graph_native/graph_native.cpp); here the graph is a
// traced torch.fx graph that Python flattens into a node table (operation
// keys, value types, leaf identities, CSR inputs). This file holds the parts
// that walk the graph: pattern matching with a one-to-one binding of
// operations, the search for non-overlapping occurrences, the order of the
// graph once accepted occurrences are replaced by region nodes (with cycle
// detection), and the structural-equality proof. Python rebuilds the torch.fx
// graph from the order and binds the region nodes to kernels.
//
// Built with g++ (no CUDA) into metal_autotune_b200/lib/libmt_graph.so.
#include "mt_graph.h"

#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

namespace {

thread_local std::string g_error;

int fail(int code, const std::string& what) {
  g_error = what;
  return code;
}

struct View {
  const mt_graph_view* v;
  int n() const { return v->n_nodes; }
  int64_t op(int i) const { return v->op[i]; }
  int64_t type(int i) const { return v->type[i]; }
  int64_t leaf(int i) const { return v->leaf[i]; }
  int in_begin(int i) const { return v->in_off[i]; }
  int in_end(int i) const { return v->in_off[i + 1]; }
  int degree(int i) const { return v->in_off[i + 1] - v->in_off[i]; }
  int input(int i, int j) const { return v->in_idx[v->in_off[i] + j]; }
};

// A table is usable when its offsets are monotone from 0 and every input
// precedes its consumer (topological order).
bool check_view(const mt_graph_view* g, const char* which) {
  if (g == nullptr || g->n_nodes < 0 || (g->n_nodes > 0 && (!g->op || !g->type || !g->leaf || !g->in_off))) {
    fail(MT_GRAPH_ERR_ARG, std::string(which) + ": null or negative-sized table");
    return false;
  }
  if (g->n_nodes == 0) return true;
  if (g->in_off[0] != 0) {
    fail(MT_GRAPH_ERR_ARG, std::string(which) + ": in_off[0] must be 0");
    return false;
  }
  for (int i = 0; i < g->n_nodes; ++i) {
    if (g->in_off[i + 1] < g->in_off[i]) {
      fail(MT_GRAPH_ERR_ARG, std::string(which) + ": in_off decreases at node " + std::to_string(i));
      return false;
    }
    if (g->in_off[i + 1] > g->in_off[i] && g->in_idx == nullptr) {
      fail(MT_GRAPH_ERR_ARG, std::string(which) + ": inputs without in_idx");
      return false;
    }
    for (int e = g->in_off[i]; e < g->in_off[i + 1]; ++e) {
      const int x = g->in_idx[e];
      if (x < 0 || x >= i) {
        fail(MT_GRAPH_ERR_ARG, std::string(which) + ": node " + std::to_string(i) + " reads node " +
                                   std::to_string(x) + " (inputs must precede their consumer)");
        return false;
      }
    }
  }
  return true;
}

// Binding state of one match attempt: pattern node -> graph node, and for
// operation nodes the reverse (graph node -> the one pattern node it stands
// for). Copied per trial; patterns are small.
struct Binding {
  std::vector<int32_t> bound;                    // [pattern nodes], -1 unbound
  std::unordered_map<int32_t, int32_t> owner;    // graph op node -> pattern node
};

// Extends `b` so that pattern node p0 stands for graph node g0, walking
// inputs pairwise. Parameters bind freely (and may share a graph node);
// other leaves must meet a graph leaf of the same identity; operations must
// agree in key, type and input count, and no graph operation may stand for
// two pattern operations.
bool match(const View& P, const View& G, const std::vector<uint8_t>& is_param, int p0, int g0, Binding& b) {
  std::vector<std::pair<int, int>> pending{{p0, g0}};
  while (!pending.empty()) {
    const auto [p, g] = pending.back();
    pending.pop_back();
    if (P.type(p) != G.type(g)) return false;
    if (b.bound[p] >= 0) {
      if (b.bound[p] != g) return false;
      continue;
    }
    if (is_param[p]) {
      b.bound[p] = g;
      continue;
    }
    if (P.op(p) == 0) {
      if (G.op(g) != 0 || G.leaf(g) != P.leaf(p)) return false;
      b.bound[p] = g;
      continue;
    }
    if (G.op(g) != P.op(p) || G.degree(g) != P.degree(p)) return false;
    const auto it = b.owner.find(g);
    if (it != b.owner.end() && it->second != p) return false;
    b.bound[p] = g;
    b.owner.emplace(g, p);
    for (int j = P.degree(p) - 1; j >= 0; --j) pending.emplace_back(P.input(p, j), G.input(g, j));
  }
  return true;
}

}  // namespace

extern "C" {

int mt_graph_version(void) { return 1; }

const char* mt_graph_error_string(void) { return g_error.c_str(); }

int mt_graph_find(const mt_graph_view* graph, const mt_graph_view* pattern, const int32_t* params,
                  int32_t n_params, const int32_t* outs, int32_t n_outs, const int32_t* anchors, int32_t* occ,
                  int32_t max_occ) {
  g_error.clear();
  if (!check_view(graph, "graph") || !check_view(pattern, "pattern")) return MT_GRAPH_ERR_ARG;
  const View G{graph}, P{pattern};
  if (n_outs <= 0 || outs == nullptr) return fail(MT_GRAPH_ERR_ARG, "a pattern needs at least one output");
  if (n_params < 0 || (n_params > 0 && params == nullptr)) return fail(MT_GRAPH_ERR_ARG, "bad parameter list");
  if (max_occ < 0 || (max_occ > 0 && occ == nullptr)) return fail(MT_GRAPH_ERR_ARG, "bad occurrence buffer");
  std::vector<uint8_t> is_param(P.n(), 0);
  for (int i = 0; i < n_params; ++i) {
    const int p = params[i];
    if (p < 0 || p >= P.n()) return fail(MT_GRAPH_ERR_ARG, "parameter index out of range");
    if (is_param[p]) return fail(MT_GRAPH_ERR_ARG, "pattern parameters must be distinct nodes");
    is_param[p] = 1;
    if (anchors && (anchors[i] < -1 || anchors[i] >= G.n()))
      return fail(MT_GRAPH_ERR_ARG, "anchor index out of range");
  }
  for (int i = 0; i < n_outs; ++i) {
    const int p = outs[i];
    if (p < 0 || p >= P.n()) return fail(MT_GRAPH_ERR_ARG, "output index out of range");
    if (P.op(p) == 0 || is_param[p])
      return fail(MT_GRAPH_ERR_ARG, "pattern outputs must be operations, not parameters or leaves");
  }

  std::unordered_map<int64_t, std::vector<int32_t>> by_op;
  for (int g = 0; g < G.n(); ++g)
    if (G.op(g) != 0) by_op[G.op(g)].push_back(g);
  auto candidates = [&](int p) -> const std::vector<int32_t>& {
    static const std::vector<int32_t> none;
    const auto it = by_op.find(P.op(p));
    return it == by_op.end() ? none : it->second;
  };

  std::vector<int32_t> owner_occ(G.n(), -1);  // graph node -> occurrence whose output it is
  Binding fixed;
  fixed.bound.assign(P.n(), -1);
  if (anchors)
    for (int i = 0; i < n_params; ++i)
      if (anchors[i] >= 0) fixed.bound[params[i]] = anchors[i];

  // Binds outs[i..n_outs-2] (the last output is bound first), trying graph
  // candidates in order and backtracking.
  auto complete = [&](auto&& self, int i, Binding& b) -> bool {
    if (i == n_outs - 1) return true;
    const int p = outs[i];
    if (b.bound[p] >= 0) {
      if (owner_occ[b.bound[p]] >= 0) return false;
      return self(self, i + 1, b);
    }
    for (const int c : candidates(p)) {
      if (owner_occ[c] >= 0) continue;
      Binding trial = b;
      if (match(P, G, is_param, p, c, trial) && self(self, i + 1, trial)) {
        b = std::move(trial);
        return true;
      }
    }
    return false;
  };

  int found = 0;
  const int last = outs[n_outs - 1];
  for (const int g : candidates(last)) {
    if (owner_occ[g] >= 0) continue;
    Binding b = fixed;
    if (!match(P, G, is_param, last, g, b)) continue;
    if (!complete(complete, 0, b)) continue;
    for (int i = 0; i < n_params; ++i)
      if (b.bound[params[i]] < 0)
        return fail(MT_GRAPH_ERR_UNUSED, "pattern parameter " + std::to_string(i) + " is not used by its outputs");
    // an occurrence must not read a value it computes itself
    bool cyclic = false;
    for (int i = 0; i < n_params && !cyclic; ++i) cyclic = b.owner.count(b.bound[params[i]]) != 0;
    if (cyclic) continue;
    bool taken = false;
    for (int i = 0; i < n_outs; ++i) taken |= owner_occ[b.bound[outs[i]]] >= 0;
    if (taken) continue;
    for (int i = 0; i < n_outs; ++i) owner_occ[b.bound[outs[i]]] = found;
    if (found < max_occ) {
      int32_t* rec = occ + static_cast<size_t>(found) * (n_params + n_outs);
      for (int i = 0; i < n_params; ++i) rec[i] = b.bound[params[i]];
      for (int i = 0; i < n_outs; ++i) rec[n_params + i] = b.bound[outs[i]];
    }
    ++found;
  }
  return found;
}

int mt_graph_order(const mt_graph_view* graph, const int32_t* roots, int32_t n_roots, const int32_t* occ,
                   int32_t n_occ, int32_t n_params, int32_t n_outs, const uint8_t* accept, int32_t* order,
                   int32_t cap) {
  g_error.clear();
  if (!check_view(graph, "graph")) return MT_GRAPH_ERR_ARG;
  const View G{graph};
  if (n_roots < 0 || (n_roots > 0 && roots == nullptr) || n_occ < 0 || n_params < 0 || n_outs <= 0 ||
      (n_occ > 0 && (occ == nullptr || accept == nullptr)) || cap < 0 || (cap > 0 && order == nullptr))
    return fail(MT_GRAPH_ERR_ARG, "bad arguments");
  const int width = n_params + n_outs;
  for (int64_t e = 0; e < static_cast<int64_t>(n_occ) * width; ++e)
    if (occ[e] < 0 || occ[e] >= G.n()) return fail(MT_GRAPH_ERR_ARG, "occurrence node out of range");
  for (int r = 0; r < n_roots; ++r)
    if (roots[r] < 0 || roots[r] >= G.n()) return fail(MT_GRAPH_ERR_ARG, "root out of range");

  // value of graph node x after the replacement: itself, or region k
  std::vector<int32_t> region_of(G.n(), -1);
  for (int k = 0; k < n_occ; ++k) {
    if (!accept[k]) continue;
    for (int j = 0; j < n_outs; ++j) {
      const int o = occ[static_cast<size_t>(k) * width + n_params + j];
      if (region_of[o] >= 0 && region_of[o] != k)
        return fail(MT_GRAPH_ERR_ARG, "a node is the output of two accepted occurrences");
      region_of[o] = k;
    }
  }
  const int n_items = G.n() + n_occ;  // items: graph nodes, then region nodes
  auto resolve = [&](int x) { return region_of[x] >= 0 ? G.n() + region_of[x] : x; };

  std::vector<uint8_t> state(n_items, 0);  // 0 new, 1 on the path, 2 emitted
  std::vector<std::pair<int, int>> stack;  // (item, next input to visit)
  int count = 0;
  auto deps = [&](int item) -> int {
    return item < G.n() ? G.degree(item) : n_params;
  };
  auto dep = [&](int item, int j) -> int {
    return item < G.n() ? resolve(G.input(item, j)) : resolve(occ[static_cast<size_t>(item - G.n()) * width + j]);
  };
  for (int r = 0; r < n_roots; ++r) {
    const int start = resolve(roots[r]);
    if (state[start] == 2) continue;
    stack.emplace_back(start, 0);
    state[start] = 1;
    while (!stack.empty()) {
      auto& [item, next] = stack.back();
      if (next < deps(item)) {
        const int d = dep(item, next++);
        if (state[d] == 1)
          return fail(MT_GRAPH_ERR_CYCLE, "graph replacement would introduce a dependency cycle");
        if (state[d] == 0) {
          state[d] = 1;
          stack.emplace_back(d, 0);
        }
        continue;
      }
      if (count >= cap) return fail(MT_GRAPH_ERR_CAPACITY, "order buffer too small");
      order[2 * count] = item < G.n() ? 0 : 1;
      order[2 * count + 1] = item < G.n() ? item : item - G.n();
      ++count;
      state[item] = 2;
      stack.pop_back();
    }
  }
  return count;
}

int mt_graph_same(const mt_graph_view* a, const int32_t* roots_a, const mt_graph_view* b, const int32_t* roots_b,
                  int32_t n_roots, char* reason, int32_t reason_len) {
  g_error.clear();
  if (!check_view(a, "first graph") || !check_view(b, "second graph")) return MT_GRAPH_ERR_ARG;
  if (n_roots < 0 || (n_roots > 0 && (roots_a == nullptr || roots_b == nullptr)))
    return fail(MT_GRAPH_ERR_ARG, "bad roots");
  const View A{a}, B{b};
  auto verdict = [&](int same, const std::string& why) {
    if (reason != nullptr && reason_len > 0) std::snprintf(reason, static_cast<size_t>(reason_len), "%s", why.c_str());
    return same;
  };
  std::vector<int32_t> ab(A.n(), -1), ba(B.n(), -1);
  std::vector<std::pair<int, int>> pending;
  for (int r = n_roots - 1; r >= 0; --r) {
    if (roots_a[r] < 0 || roots_a[r] >= A.n() || roots_b[r] < 0 || roots_b[r] >= B.n())
      return fail(MT_GRAPH_ERR_ARG, "root out of range");
    pending.emplace_back(roots_a[r], roots_b[r]);
  }
  while (!pending.empty()) {
    const auto [x, y] = pending.back();
    pending.pop_back();
    if (ab[x] >= 0) {
      if (ab[x] != y) return verdict(0, "shared node duplicated (first graph node " + std::to_string(x) + ")");
      continue;
    }
    if (ba[y] >= 0 && ba[y] != x)
      return verdict(0, "distinct nodes merged (second graph node " + std::to_string(y) + ")");
    ab[x] = y;
    ba[y] = x;
    const std::string at = " at nodes " + std::to_string(x) + " / " + std::to_string(y);
    if (A.type(x) != B.type(y)) return verdict(0, "shape or dtype" + at);
    if ((A.op(x) == 0) != (B.op(y) == 0)) return verdict(0, "operation versus leaf" + at);
    if (A.op(x) == 0) {
      if (A.leaf(x) != B.leaf(y)) return verdict(0, "different leaf" + at);
      continue;
    }
    if (A.op(x) != B.op(y)) return verdict(0, "operation mismatch" + at);
    if (A.degree(x) != B.degree(y)) return verdict(0, "input count" + at);
    for (int j = A.degree(x) - 1; j >= 0; --j) pending.emplace_back(A.input(x, j), B.input(y, j));
  }
  return verdict(1, "same operations, attributes, leaves and sharing");
}

}  // extern "C"
