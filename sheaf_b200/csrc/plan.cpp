// Planner: dead-code elimination, fusion clustering, GEMM operand views,
// split-reduction sizing and the liveness-based arena layout.
//
// Fusion model.  Every live value is one of
//   * materialized: a parameter, a dense constant (uploaded at load), or the
//     root of a step (written to memory);
//   * duplicable: splat constants, iota and the pure index maps (broadcast,
//     reshape, transpose, slice, reverse).  These are never written to memory;
//     each consumer cluster re-evaluates them from coordinates;
//   * fused: an expression node evaluated inside the single cluster that
//     consumes it.
// A non-duplicable node joins its consumer's cluster when all of its uses (seen
// through duplicable nodes) lie in one cluster and none of them is a GEMM
// operand or a gather table; otherwise it becomes the root of a new cluster.
// Reductions, dot_generals and returned values are always roots.
#include "plan.h"

#include <algorithm>
#include <cstdlib>
#include <cmath>
#include <functional>
#include <map>
#include <set>
#include <sstream>
#include <stdexcept>

#include "codegen.h"
#include "kernels/kernels.h"

namespace sb {

std::vector<int64_t> row_major(const std::vector<int64_t>& shape) {
  std::vector<int64_t> s(shape.size(), 1);
  for (int i = (int)shape.size() - 2; i >= 0; --i) s[i] = s[i + 1] * shape[i + 1];
  return s;
}

// numpy-style no-copy reshape of a strided view; returns false if impossible.
bool reshape_view(const std::vector<int64_t>& oshape, const std::vector<int64_t>& ostr,
                  const std::vector<int64_t>& nshape, std::vector<int64_t>* nstr) {
  std::vector<int64_t> os, ost;
  for (size_t i = 0; i < oshape.size(); ++i)
    if (oshape[i] != 1) { os.push_back(oshape[i]); ost.push_back(ostr[i]); }
  nstr->assign(nshape.size(), 0);
  size_t oi = 0, ni = 0;
  int on = (int)os.size(), nn = (int)nshape.size();
  while (ni < (size_t)nn && oi < (size_t)on) {
    if (nshape[ni] == 1) { (*nstr)[ni] = 0; ++ni; continue; }
    int64_t np = nshape[ni], op = os[oi];
    size_t nj = ni + 1, oj = oi + 1;
    while (np != op) {
      if (np < op) {
        if (nj >= (size_t)nn) return false;
        np *= nshape[nj++];
      } else {
        if (oj >= (size_t)on) return false;
        op *= os[oj++];
      }
    }
    for (size_t k = oi; k + 1 < oj; ++k)
      if (ost[k] != ost[k + 1] * os[k + 1]) return false;
    (*nstr)[nj - 1] = ost[oj - 1];
    for (size_t k = nj - 1; k > ni; --k) (*nstr)[k - 1] = (*nstr)[k] * nshape[k];
    ni = nj;
    oi = oj;
  }
  for (; ni < (size_t)nn; ++ni) {
    if (nshape[ni] != 1) return false;
    (*nstr)[ni] = 0;
  }
  return oi == (size_t)on;
}

namespace {

constexpr int kDup = -2;   // duplicable (never materialized)
constexpr int kConst = -3; // dense constant buffer
constexpr int kParam = -4;
constexpr int kAbsorbed = -5;  // batched dot_general folded into the GEMM of its batch reduction

bool is_dup_kind(const Op& op) {
  switch (op.kind) {
    case OpKind::BroadcastInDim: case OpKind::Reshape: case OpKind::Transpose:
    case OpKind::Slice: case OpKind::Reverse: case OpKind::Iota: case OpKind::StridedView:
      return true;
    case OpKind::Constant:
      return op.values.size() == 1;
    default:
      return false;
  }
}

[[noreturn]] void fail(const Op& op, const std::string& msg) {
  throw std::runtime_error("line " + std::to_string(op.line) + " (" + opkind_name(op.kind) + "): " + msg);
}


struct Planner {
  const Function& f;
  Precision prec;
  int NV, P;
  std::vector<char> live;
  std::vector<std::vector<std::pair<int, int>>> consumers;  // value -> (op index, slot)
  std::vector<int> cluster;  // root id, kDup, kConst, kParam
  std::set<int> forced;
  std::vector<char> returned;

  Planner(const Function& fn, Precision p) : f(fn), prec(p) {
    NV = f.num_values();
    P = (int)f.params.size();
  }

  const Op* producer(int v) const { return f.producer[v] >= 0 ? &f.ops[f.producer[v]] : nullptr; }

  void liveness() {
    live.assign(NV, 0);
    returned.assign(NV, 0);
    for (int r : f.returns) { live[r] = 1; returned[r] = 1; }
    for (int i = (int)f.ops.size() - 1; i >= 0; --i) {
      const Op& op = f.ops[i];
      if (!live[op.result]) continue;
      for (int o : op.operands) live[o] = 1;
    }
    consumers.assign(NV, {});
    for (int i = 0; i < (int)f.ops.size(); ++i) {
      const Op& op = f.ops[i];
      if (!live[op.result]) continue;
      for (int s = 0; s < (int)op.operands.size(); ++s) consumers[op.operands[s]].push_back({i, s});
      // the sort kernel reads dense buffers: its operands are materialized
      if (op.kind == OpKind::SortPairs || op.kind == OpKind::ScatterAddRows)
        for (int o : op.operands) forced.insert(o);
    }
    find_batch_reduced_dots();
  }

  // reduce(add, init 0) over a batch dimension of a dot_general that has no
  // other use: sum_b A_b @ B_b is one GEMM whose contraction also runs over b.
  // This is how weight gradients of 3-D activations arrive
  // (transpose(x) @ adj, then sum_to_shape over the batch).
  std::map<int, int> fused_dot;  // reduce result -> dot op index
  void find_batch_reduced_dots() {
    for (int i = 0; i < (int)f.ops.size(); ++i) {
      const Op& r = f.ops[i];
      if (!live[r.result] || r.kind != OpKind::Reduce || r.body != ReduceBody::Add || r.dims.size() != 1) continue;
      int x = r.operands[0];
      const Op* d = producer(x);
      if (!d || d->kind != OpKind::DotGeneral || returned[x] || consumers[x].size() != 1) continue;
      const Op* init = producer(r.operands[1]);
      if (!init || init->kind != OpKind::Constant || init->values.size() != 1 || init->values[0] != 0.0) continue;
      if (r.dims[0] >= (int64_t)d->lb.size()) continue;
      fused_dot[r.result] = f.producer[x];
    }
  }

  // The dot_general a GEMM step computes: the op itself, or for a fused batch
  // reduction the absorbed dot with the reduced batch dim moved into the
  // contraction (outermost, so it merges with the contracting dims).
  Op gemm_op(const Op& op) const {
    auto it = fused_dot.find(op.result);
    if (it == fused_dot.end()) return op;
    Op d = f.ops[it->second];
    size_t bd = (size_t)op.dims[0];
    int64_t l = d.lb[bd], r = d.rb[bd];
    d.lb.erase(d.lb.begin() + bd);
    d.rb.erase(d.rb.begin() + bd);
    d.lc.insert(d.lc.begin(), l);
    d.rc.insert(d.rc.begin(), r);
    d.type = op.type;
    d.result = op.result;
    return d;
  }
  // True when every use of v (seen through index maps) is a GEMM operand.
  // Row groups: does the cluster of step root `member` (evaluated from node n
  // at coordinate class cls: 0 = [rows..., C] element, 1 = row, 2 = other)
  // read each value of `inside` (an earlier member's output -> its class)
  // only at its own row?  Index maps that keep the row: same-shape operands,
  // reshapes that keep (rows, C) or the row count, broadcasts of a row vector
  // along C, and the innermost-dim reduction of a [rows..., C] operand.
  bool row_local(int n, int cls, int member, const std::map<int, int>& inside, int64_t R, int64_t C,
                 std::set<std::pair<int, int>>& seen) const {
    if (!seen.insert({n, cls}).second) return true;
    const int cl = cluster[n];
    if (cl == kParam || cl == kConst || (cl == n && n != member)) {
      auto it = inside.find(n);
      return it == inside.end() || (cls != 2 && it->second == cls);
    }
    const Op* op = producer(n);
    if (!op) return true;
    const auto& os = f.value_types[n].shape;
    auto visit_all = [&](int c2) {
      for (int o : op->operands)
        if (!row_local(o, c2, member, inside, R, C, seen)) return false;
      return true;
    };
    if (is_elementwise(op->kind)) {
      for (int o : op->operands) {
        const int oc = f.value_types[o].shape == os ? cls : 2;
        if (!row_local(o, oc, member, inside, R, C, seen)) return false;
      }
      return true;
    }
    switch (op->kind) {
      case OpKind::Constant: case OpKind::Iota:
        return true;
      case OpKind::Reduce: {
        const auto& is = f.value_types[op->operands[0]].shape;
        bool colred = n == member && is.size() >= 2 && op->dims.size() == is.size() - 1 && is.back() == C &&
                      f.value_types[op->operands[0]].numel() == R * C;
        for (size_t d = 0; colred && d + 1 < is.size(); ++d) colred = op->dims[d] == (int64_t)d;
        if (colred) {
          if (!row_local(op->operands[0], 0, member, inside, R, C, seen)) return false;
          return row_local(op->operands[1], 2, member, inside, R, C, seen);
        }
        const bool rowred = cls == 1 && op->dims.size() == 1 && !is.empty() && op->dims[0] == (int64_t)is.size() - 1 &&
                            is.back() == C && f.value_types[n].numel() == R;
        if (!row_local(op->operands[0], rowred ? 0 : 2, member, inside, R, C, seen)) return false;
        return row_local(op->operands[1], 2, member, inside, R, C, seen);
      }
      case OpKind::Reshape: {
        const Type& it = f.value_types[op->operands[0]];
        int oc = 2;
        if (cls == 0 && !it.shape.empty() && !os.empty() && it.shape.back() == C && os.back() == C) oc = 0;
        if (cls == 1 && it.numel() == R) oc = 1;
        return row_local(op->operands[0], oc, member, inside, R, C, seen);
      }
      case OpKind::BroadcastInDim: {
        const Type& it = f.value_types[op->operands[0]];
        int oc = 2;
        if (it.shape == os) {
          oc = cls;
        } else if ((cls == 0 || cls == 1) && it.numel() == R) {
          // non-unit input dims map in order onto equal row dims of the output
          bool ok = true;
          int64_t last = -1;
          for (size_t i = 0; i < it.shape.size(); ++i) {
            if (it.shape[i] == 1) continue;
            const int64_t d = op->dims[i];
            ok = ok && d > last && os[d] == it.shape[i] && (cls == 1 || d + 1 < (int64_t)os.size());
            last = d;
          }
          if (ok) oc = 1;
        }
        return row_local(op->operands[0], oc, member, inside, R, C, seen);
      }
      default:
        return visit_all(2);
    }
  }

  bool only_gemm_consumers(int v) const {
    if (returned[v]) return false;
    for (auto [oi, slot] : consumers[v]) {
      const Op& c = f.ops[oi];
      if (c.kind == OpKind::DotGeneral || is_attention(c.kind)) continue;
      if (cluster[c.result] == kDup && !returned[c.result]) {
        if (!only_gemm_consumers(c.result)) return false;
        continue;
      }
      return false;
    }
    return !consumers[v].empty();
  }
  bool is_gemm_root(const Op& op) const {
    if (op.kind == OpKind::DotGeneral) return cluster.empty() || cluster[op.result] != kAbsorbed;
    return op.kind == OpKind::Reduce && fused_dot.count(op.result);
  }

  void collect(int v, std::set<int>& cs, bool& blocked, std::set<int>& seen) {
    for (auto [oi, slot] : consumers[v]) {
      const Op& c = f.ops[oi];
      if (c.kind == OpKind::DotGeneral || is_attention(c.kind) || c.kind == OpKind::SortPairs ||
          c.kind == OpKind::ScatterAddRows) {
        blocked = true;
        continue;
      }
      if (c.kind == OpKind::Gather && slot == 0) { blocked = true; continue; }
      int cv = c.result;
      if (cluster[cv] == kDup) {
        if (seen.insert(cv).second) collect(cv, cs, blocked, seen);
      } else {
        cs.insert(cluster[cv]);
      }
    }
  }

  // Rematerialization.  An element-wise value used by several clusters is
  // recomputed inside each of them instead of being written and re-read, when
  // the recomputation is cheap: at most kRematOps element-wise ops (at most
  // two transcendental) down to at most three values that are materialized
  // anyway, and every consumer reads it at its own shape (no broadcast that
  // would repeat the work).  Typical cases: the tanh term of GELU and the
  // normalized input of layer norm, which the reverse pass would otherwise
  // read back from HBM.
  static constexpr int kRematOps = 16;
  static bool transcendental(OpKind k) {
    return k == OpKind::Tanh || k == OpKind::Exp || k == OpKind::Log || k == OpKind::Sin || k == OpKind::Cos ||
           k == OpKind::Logistic || k == OpKind::Pow || k == OpKind::Sqrt || k == OpKind::Rsqrt;
  }
  bool remat_cone(int u, int& ops, int& trans, std::set<int>& leaves, std::set<int>& seen) const {
    if (!seen.insert(u).second) return true;
    const Op* p = producer(u);
    // a value already made a root, or (not yet decided: it comes earlier in
    // the program) one with several uses, is read, not recomputed
    const bool shared = p && (cluster[u] == u || (cluster[u] == -1 && consumers[u].size() > 1 && !is_dup_kind(*p)));
    if (!p || returned[u] || forced.count(u) || shared || p->kind == OpKind::Reduce || p->kind == OpKind::DotGeneral ||
        is_attention(p->kind) || (p->kind == OpKind::Constant && p->values.size() != 1)) {
      leaves.insert(u);
      return leaves.size() <= 3;
    }
    if (p->kind == OpKind::Constant || p->kind == OpKind::Iota) return true;
    if (is_dup_kind(*p)) return remat_cone(p->operands[0], ops, trans, leaves, seen);
    if (!is_elementwise(p->kind)) return false;
    if (++ops > kRematOps || (transcendental(p->kind) && ++trans > 2)) return false;
    for (int o : p->operands)
      if (!remat_cone(o, ops, trans, leaves, seen)) return false;
    return true;
  }
  bool same_shape_uses(int v, int depth = 0) const {
    if (depth > 8) return false;
    for (auto [oi, slot] : consumers[v]) {
      const Op& c = f.ops[oi];
      if (!is_dup_kind(c)) continue;
      if (c.kind != OpKind::Reshape && c.kind != OpKind::Transpose && c.kind != OpKind::Slice) return false;
      if (!same_shape_uses(c.result, depth + 1)) return false;
    }
    return true;
  }
  bool rematerializable(int v) const {
    const Op* p = producer(v);
    if (!p || !is_elementwise(p->kind) || returned[v] || f.value_types[v].numel() < (1 << 16)) return false;
    if (!same_shape_uses(v)) return false;
    int ops = 0, trans = 0;
    std::set<int> leaves, seen;
    return remat_cone(v, ops, trans, leaves, seen);
  }

  // The cone a rematerialized value really has once every value is decided:
  // kDup nodes are recomputed (followed), everything else is read.  A value
  // whose cone grew past the limits (its producers were assumed to be read
  // but were themselves rematerialized) becomes a root; true if any did.
  bool real_cone(int u, int& ops, int& trans, std::set<int>& leaves, std::set<int>& seen) const {
    if (!seen.insert(u).second) return true;
    const Op* p = producer(u);
    if (!p || cluster[u] != kDup) {
      leaves.insert(u);
      return leaves.size() <= 3;
    }
    if (p->kind == OpKind::Constant || p->kind == OpKind::Iota) return true;
    if (is_elementwise(p->kind)) {
      if (++ops > kRematOps || (transcendental(p->kind) && ++trans > 2)) return false;
    }
    for (int o : p->operands)
      if (!real_cone(o, ops, trans, leaves, seen)) return false;
    return true;
  }
  bool validate_remat() {
    bool changed = false;
    for (const Op& op : f.ops) {
      const int v = op.result;
      if (!live[v] || cluster[v] != kDup || !is_elementwise(op.kind)) continue;
      int ops = 0, trans = 0;
      std::set<int> leaves, seen;
      if (!real_cone(v, ops, trans, leaves, seen)) {
        forced.insert(v);
        changed = true;
      }
    }
    return changed;
  }

  void clusterize() {
    cluster.assign(NV, -1);
    for (int p = 0; p < P; ++p) cluster[p] = kParam;
    for (int i = (int)f.ops.size() - 1; i >= 0; --i) {
      const Op& op = f.ops[i];
      int v = op.result;
      if (!live[v]) continue;
      if (op.kind == OpKind::Constant && op.values.size() != 1) { cluster[v] = kConst; continue; }
      bool absorbed = false;
      for (auto& [rv, di] : fused_dot) if (di == i) absorbed = true;
      if (absorbed) { cluster[v] = kAbsorbed; continue; }
      if (returned[v] || forced.count(v) || op.kind == OpKind::Reduce || op.kind == OpKind::DotGeneral ||
          is_attention(op.kind) || op.kind == OpKind::SortPairs || op.kind == OpKind::ScatterAddRows) {
        cluster[v] = v;
        continue;
      }
      if (is_dup_kind(op)) { cluster[v] = kDup; continue; }
      std::set<int> cs, seen;
      bool blocked = false;
      collect(v, cs, blocked, seen);
      if (!blocked && cs.size() == 1) cluster[v] = *cs.begin();
      else if (!blocked && cs.size() > 1 && rematerializable(v)) cluster[v] = kDup;
      else cluster[v] = v;
    }
  }

  // Reduction epilogues.  A row reduction X (trailing dims) whose every use
  // is an element-wise op of one loop cluster R (directly or through reshapes
  // that only add or drop unit dims), with R of X's shape up to unit dims and
  // X reached from R through element-wise ops and such reshapes only, is
  // computed inside R's kernel: the reduction runs per output element of R
  // and R's expression is evaluated on the result (layer-norm statistics
  // followed by their scalar arithmetic become one kernel).  cluster[X]
  // becomes R; epilogue_of[R] = X.
  std::map<int, int> epilogue_of;
  static std::vector<int64_t> nonunit(const std::vector<int64_t>& sh) {
    std::vector<int64_t> r;
    for (int64_t d : sh)
      if (d != 1) r.push_back(d);
    return r;
  }
  // reshape / broadcast_in_dim that only inserts or removes unit dims
  bool unit_map(int v) const {
    const Op* p = producer(v);
    if (!p || cluster[v] != kDup) return false;
    if (p->kind != OpKind::Reshape && p->kind != OpKind::BroadcastInDim) return false;
    const auto& in = f.value_types[p->operands[0]].shape;
    if (nonunit(in) != nonunit(p->type.shape)) return false;
    if (p->kind == OpKind::BroadcastInDim)
      for (size_t i = 1; i < p->dims.size(); ++i)
        if (p->dims[i] <= p->dims[i - 1]) return false;
    return true;
  }
  // every use of v is an element-wise op of one cluster (*R), possibly through unit maps
  bool uses_in_one_cluster(int v, int* R, int depth = 0) const {
    if (depth > 8 || returned[v] || consumers[v].empty()) return false;
    for (auto [oi, slot] : consumers[v]) {
      const Op& c = f.ops[oi];
      if (unit_map(c.result)) {
        if (!uses_in_one_cluster(c.result, R, depth + 1)) return false;
        continue;
      }
      const int cr = cluster[c.result];
      if (!is_elementwise(c.kind) || cr < 0 || (*R >= 0 && cr != *R)) return false;
      *R = cr;
    }
    return true;
  }
  bool reaches_elementwise_only(int u, int R, int X, std::set<int>& seen, bool& hit) const {
    if (!seen.insert(u).second) return true;
    const Op* p = producer(u);
    if (!p) return true;
    for (int o : p->operands) {
      if (o == X) { hit = true; continue; }
      if (cluster[o] == R) {
        const Op* q = producer(o);
        if (!q || !is_elementwise(q->kind)) return false;
        if (!reaches_elementwise_only(o, R, X, seen, hit)) return false;
      } else if (unit_map(o)) {
        if (!reaches_elementwise_only(o, R, X, seen, hit)) return false;
      } else if (cluster[o] == kDup) {
        // X must not be read through any other index map
        std::set<int> seen2;
        if (reads_value(o, R, X, seen2)) return false;
      }
    }
    return true;
  }
  // True when evaluating u inside cluster R reads X.
  bool reads_value(int u, int R, int X, std::set<int>& seen) const {
    if (u == X) return true;
    if (!seen.insert(u).second || (cluster[u] != kDup && cluster[u] != R)) return false;
    const Op* p = producer(u);
    if (!p) return false;
    for (int o : p->operands)
      if (reads_value(o, R, X, seen)) return true;
    return false;
  }
  // The single element-wise use of v (seen through unit maps), or -1.
  int single_elementwise_use(int v) const {
    int u = v, depth = 0;
    for (;;) {
      if (returned[u] || consumers[u].size() != 1 || ++depth > 8) return -1;
      const Op& c = f.ops[consumers[u][0].first];
      if (unit_map(c.result)) { u = c.result; continue; }
      return is_elementwise(c.kind) ? c.result : -1;
    }
  }
  // Returns true when it made a value a root (the clustering must be redone):
  // the top T of a row reduction's per-row element-wise chain (same shape up
  // to unit dims, one use per step), when T's cluster is wider (T is read
  // through a broadcast), so that the per-row arithmetic runs once per row in
  // the reduction's epilogue instead of once per element of the consumer.
  bool absorb_reduce_epilogues() {
    bool changed = false;
    epilogue_of.clear();
    for (const Op& x : f.ops) {
      const int X = x.result;
      if (!live[X] || x.kind != OpKind::Reduce || cluster[X] != X || returned[X] || forced.count(X) ||
          fused_dot.count(X))
        continue;
      const int r = (int)f.value_types[x.operands[0]].shape.size();
      std::vector<int64_t> rd(x.dims.begin(), x.dims.end());
      std::sort(rd.begin(), rd.end());
      bool trailing = !rd.empty();
      for (size_t i = 0; i < rd.size(); ++i)
        if (rd[rd.size() - 1 - i] != r - 1 - (int64_t)i) trailing = false;
      if (!trailing) continue;
      int R = -1;
      if (!uses_in_one_cluster(X, &R) || R < 0 || epilogue_of.count(R)) continue;
      const Op* ro = producer(R);
      if (ro && is_elementwise(ro->kind) && nonunit(f.value_types[R].shape) != nonunit(f.value_types[X].shape)) {
        const auto xs = nonunit(f.value_types[X].shape);
        int t = X;
        for (int u = single_elementwise_use(X); u >= 0 && cluster[u] == R && nonunit(f.value_types[u].shape) == xs &&
                                                f.value_types[u].dtype == DType::F32;
             u = single_elementwise_use(u))
          t = u;
        if (t != X && !forced.count(t)) {
          forced.insert(t);
          changed = true;
        }
        continue;
      }
      if (!ro || !is_elementwise(ro->kind) || nonunit(f.value_types[R].shape) != nonunit(f.value_types[X].shape) ||
          f.value_types[R].dtype != DType::F32 || f.value_types[X].dtype != DType::F32)
        continue;
      std::set<int> seen;
      bool hit = false;
      if (!reaches_elementwise_only(R, R, X, seen, hit) || !hit) continue;
      epilogue_of[R] = X;
      cluster[X] = R;
    }
    return changed;
  }

  bool materialized(int v) const { return cluster[v] == kParam || cluster[v] == kConst || cluster[v] == v; }

  // View of v over a materialized buffer, through duplicable index maps.
  bool view_of(int v, View* out) {
    if (materialized(v)) {
      out->value = v;
      out->offset = 0;
      out->shape = f.value_types[v].shape;
      out->strides = row_major(out->shape);
      return true;
    }
    const Op* op = producer(v);
    if (!op || cluster[v] != kDup) return false;
    View in;
    switch (op->kind) {
      case OpKind::Transpose: {
        if (!view_of(op->operands[0], &in)) return false;
        *out = in;
        out->shape = op->type.shape;
        for (size_t i = 0; i < op->dims.size(); ++i) out->strides[i] = in.strides[op->dims[i]];
        return true;
      }
      case OpKind::BroadcastInDim: {
        if (!view_of(op->operands[0], &in)) return false;
        *out = in;
        out->shape = op->type.shape;
        out->strides.assign(out->shape.size(), 0);
        for (size_t i = 0; i < op->dims.size(); ++i)
          if (in.shape[i] == out->shape[op->dims[i]]) out->strides[op->dims[i]] = in.strides[i];
        return true;
      }
      case OpKind::Slice: {
        if (!view_of(op->operands[0], &in)) return false;
        *out = in;
        out->shape = op->type.shape;
        for (size_t i = 0; i < in.shape.size(); ++i) {
          out->offset += op->a0[i] * in.strides[i];
          out->strides[i] = in.strides[i] * op->a2[i];
        }
        return true;
      }
      case OpKind::Reverse: {
        if (!view_of(op->operands[0], &in)) return false;
        *out = in;
        for (auto d : op->dims) {
          out->offset += (in.shape[d] - 1) * in.strides[d];
          out->strides[d] = -in.strides[d];
        }
        return true;
      }
      case OpKind::Reshape: {
        if (!view_of(op->operands[0], &in)) return false;
        std::vector<int64_t> ns;
        if (!reshape_view(in.shape, in.strides, op->type.shape, &ns)) return false;
        *out = in;
        out->shape = op->type.shape;
        out->strides = ns;
        return true;
      }
      case OpKind::StridedView: {
        // offsets and strides address the operand's row-major layout
        if (!view_of(op->operands[0], &in)) return false;
        const auto rm = row_major(in.shape);
        for (size_t i = 0; i < in.shape.size(); ++i)
          if (in.shape[i] != 1 && in.strides[i] != rm[i]) return false;
        out->value = in.value;
        out->offset = in.offset + op->a0[0];
        out->shape = op->type.shape;
        out->strides = op->a2;
        return true;
      }
      default:
        return false;
    }
  }

  // Merges dims `ds` (in order) of a view into one extent/stride; false if not mergeable.
  static bool merge(const View& v, const std::vector<int64_t>& ds, int64_t* ext, int64_t* str) {
    *ext = 1;
    *str = 0;
    std::vector<int64_t> keep;
    for (auto d : ds) if (v.shape[d] != 1) keep.push_back(d);
    for (auto d : ds) *ext *= v.shape[d];
    if (keep.empty()) { *str = 0; return true; }
    for (size_t i = 0; i + 1 < keep.size(); ++i)
      if (v.strides[keep[i]] != v.strides[keep[i + 1]] * v.shape[keep[i + 1]]) return false;
    *str = v.strides[keep.back()];
    return true;
  }

  // Tries to describe a dot_general as a strided batched GEMM.
  // Materializes the deepest value of an index-map chain that has no strided
  // view, so the maps above it (e.g. a transpose feeding a GEMM) stay views.
  void force_for_view(int v) {
    const Op* op = producer(v);
    if (op && cluster[v] == kDup && op->kind == OpKind::StridedView) {
      // a strided view needs a row-major operand: materialize the operand
      if (!materialized(op->operands[0])) {
        forced.insert(op->operands[0]);
        return;
      }
    }
    if (op && cluster[v] == kDup && op->kind != OpKind::Iota && op->kind != OpKind::Constant) {
      View in;
      if (!view_of(op->operands[0], &in)) {
        force_for_view(op->operands[0]);
        return;
      }
    }
    forced.insert(v);
  }

  bool gemm_of(const Op& root, GemmDesc* g) {
    const Op op = gemm_op(root);
    View a, b;
    bool ok = true;
    if (!view_of(op.operands[0], &a)) { force_for_view(op.operands[0]); ok = false; }
    if (!view_of(op.operands[1], &b)) { force_for_view(op.operands[1]); ok = false; }
    if (!ok) return false;
    int ra = (int)a.shape.size(), rb = (int)b.shape.size();
    std::vector<int64_t> af, bf;
    for (int d = 0; d < ra; ++d)
      if (!std::count(op.lb.begin(), op.lb.end(), d) && !std::count(op.lc.begin(), op.lc.end(), d)) af.push_back(d);
    for (int d = 0; d < rb; ++d)
      if (!std::count(op.rb.begin(), op.rb.end(), d) && !std::count(op.rc.begin(), op.rc.end(), d)) bf.push_back(d);
    int64_t e1 = 0, e2 = 0;
    bool a_ok = merge(a, op.lb, &g->batch, &g->sab) && merge(a, af, &g->M, &g->sam) &&
                merge(a, op.lc, &g->K, &g->sak);
    bool b_ok = merge(b, op.rb, &e1, &g->sbb) && merge(b, op.rc, &e2, &g->sbk) && merge(b, bf, &g->N, &g->sbn);
    if (!a_ok || !b_ok) {
      // Materialize the operand whose dims do not merge (contiguous in its own
      // dim order).  A batch reduction that still does not merge stays a
      // batched GEMM followed by a reduction.
      bool pending = false;  // an operand will be materialized on the next pass
      if (!a_ok && !materialized(op.operands[0])) { forced.insert(op.operands[0]); pending = true; }
      if (!b_ok && !materialized(op.operands[1])) { forced.insert(op.operands[1]); pending = true; }
      if (pending) return false;
      if (fused_dot.erase(root.result)) return false;
      fail(op, "dot_general operand layout is not expressible as a strided batched GEMM");
    }
    if (e1 != g->batch || e2 != g->K) fail(op, "internal: dot_general extents disagree");
    g->a = a;
    g->b = b;
    return true;
  }

  // Views of an attention op's operands.  The [B,H,T,64] operands are read by
  // TMA or 16-byte loads: unit stride on the head dim, the other strides and
  // the offset multiples of 4 elements.  An operand whose view does not qualify
  // is materialized (row-major) on the next pass.
  bool attn_of(const Op& op, AttnDesc* d) {
    d->kind = op.kind;
    d->in.clear();
    const auto& qs = f.value_types[op.operands[0]].shape;
    d->B = qs[0];
    d->H = qs[1];
    d->T = qs[2];
    d->scale = op.values.empty() ? 1.0 : op.values[0];
    d->causal = op.axis != 0;
    bool ok = true;
    for (int o : op.operands) {
      View w;
      if (!view_of(o, &w)) {
        force_for_view(o);
        ok = false;
        continue;
      }
      if (w.shape.size() == 4) {
        bool good = w.strides[3] == 1 && w.offset % 4 == 0;
        for (int i = 0; i < 3; ++i) {
          if (w.shape[i] == 1) w.strides[i] = 4;  // any 16-byte multiple: the index is always 0
          good = good && w.strides[i] > 0 && w.strides[i] % 4 == 0;
        }
        if (!good) {
          if (materialized(o)) fail(op, "internal: attention operand layout");
          forced.insert(o);
          ok = false;
          continue;
        }
      }
      d->in.push_back(w);
    }
    return ok;
  }
};

// Shape/attribute consistency of every op.  Kernels index buffers from these
// shapes, so a module that fails here never reaches the GPU.
void verify(const Function& f) {
  auto T = [&](int v) -> const Type& { return f.value_types[v]; };
  for (const Op& op : f.ops) {
    const auto& rs = op.type.shape;
    int rr = (int)rs.size();
    auto need = [&](bool c, const char* what) {
      if (!c) fail(op, std::string("malformed op: ") + what);
    };
    for (auto d : rs) need(d >= 0, "negative extent");
    if (is_elementwise(op.kind) && op.kind != OpKind::Select && op.kind != OpKind::Clamp) {
      for (int o : op.operands) need(T(o).shape == rs, "operand shape differs from result shape");
    }
    switch (op.kind) {
      case OpKind::Constant:
        need(op.values.size() == 1 || (int64_t)op.values.size() == op.type.numel(), "constant payload size");
        break;
      case OpKind::ScatterAddRows: {
        const Type& ix = T(op.operands[0]);
        const Type& ad = T(op.operands[1]);
        need(op.operands.size() == 2 && rs.size() == 2 && !ad.shape.empty() && ad.shape.back() == rs[1] &&
                 ix.numel() * rs[1] == ad.numel() && (ix.dtype == DType::F32 || ix.dtype == DType::I32) &&
                 ad.dtype == DType::F32 && op.type.dtype == DType::F32,
             "scatter_add_rows operand shapes");
        break;
      }
      case OpKind::SortPairs:
        need(op.operands.size() == 2 && T(op.operands[0]).shape == T(op.operands[1]).shape && !rs.empty() &&
                 rs.back() == 2 * T(op.operands[0]).shape.back(),
             "sort operand / packed result shapes");
        break;
      case OpKind::Bitcast: {
        const DType a = T(op.operands[0]).dtype, b = op.type.dtype;
        auto w32 = [](DType t) { return t == DType::F32 || t == DType::I32; };
        need(a == b || (w32(a) && w32(b)), "bitcast_convert between f32 and i32 only");
        break;
      }
      case OpKind::Select:
        need(T(op.operands[0]).shape == rs || T(op.operands[0]).shape.empty(), "select predicate shape");
        need(T(op.operands[1]).shape == rs && T(op.operands[2]).shape == rs, "select operand shapes");
        break;
      case OpKind::Clamp:
        need(T(op.operands[1]).shape == rs, "clamp operand shape");
        for (int k : {0, 2}) need(T(op.operands[k]).shape == rs || T(op.operands[k]).shape.empty(), "clamp bound shape");
        break;
      case OpKind::BroadcastInDim: {
        const auto& is = T(op.operands[0]).shape;
        need(op.dims.size() == is.size(), "broadcast dims arity");
        for (size_t i = 0; i < is.size(); ++i) {
          need(op.dims[i] >= 0 && op.dims[i] < rr, "broadcast dim out of range");
          if (op.dims[i] >= 0 && op.dims[i] < rr) need(is[i] == 1 || is[i] == rs[op.dims[i]], "broadcast extent");
        }
        break;
      }
      case OpKind::Reshape:
        need(T(op.operands[0]).numel() == op.type.numel(), "reshape element count");
        break;
      case OpKind::Transpose: {
        const auto& is = T(op.operands[0]).shape;
        need(op.dims.size() == is.size() && (int)is.size() == rr, "transpose arity");
        std::vector<int> seen(rr, 0);
        for (int i = 0; i < rr; ++i) {
          need(op.dims[i] >= 0 && op.dims[i] < rr && !seen[op.dims[i]]++, "transpose permutation");
          need(rs[i] == is[op.dims[i]], "transpose extent");
        }
        break;
      }
      case OpKind::Iota:
        need(op.axis >= 0 && op.axis < rr, "iota dim");
        break;
      case OpKind::StridedView: {
        need(op.operands.size() == 1 && op.a0.size() == 1 && (int)op.a2.size() == rr, "strided view arity");
        if (op.operands.size() != 1 || op.a0.size() != 1 || (int)op.a2.size() != rr) break;
        int64_t hi = op.a0[0];
        bool empty = false;
        for (int i = 0; i < rr; ++i) {
          need(op.a2[i] >= 0, "strided view stride");
          if (rs[i] == 0) empty = true;
          else hi += (rs[i] - 1) * op.a2[i];
        }
        need(op.a0[0] >= 0 && (empty || hi < T(op.operands[0]).numel()), "strided view bounds");
        need(T(op.operands[0]).dtype == op.type.dtype, "strided view element type");
        break;
      }
      case OpKind::Slice: {
        const auto& is = T(op.operands[0]).shape;
        need(op.a0.size() == is.size() && op.a1.size() == is.size() && op.a2.size() == is.size() &&
                 (int)is.size() == rr, "slice arity");
        for (int i = 0; i < rr; ++i) {
          need(op.a2[i] >= 1 && op.a0[i] >= 0 && op.a0[i] <= op.a1[i] && op.a1[i] <= is[i], "slice bounds");
          need(rs[i] == (op.a1[i] - op.a0[i] + op.a2[i] - 1) / op.a2[i], "slice extent");
        }
        break;
      }
      case OpKind::Pad: {
        const auto& is = T(op.operands[0]).shape;
        need(T(op.operands[1]).shape.empty(), "pad value must be a scalar");
        need(op.a0.size() == is.size() && op.a1.size() == is.size() && op.a2.size() == is.size() &&
                 (int)is.size() == rr, "pad arity");
        for (int i = 0; i < rr; ++i) {
          need(op.a2[i] >= 0, "negative interior padding");
          need(rs[i] == op.a0[i] + op.a1[i] + is[i] + std::max<int64_t>(is[i] - 1, 0) * op.a2[i], "pad extent");
        }
        break;
      }
      case OpKind::Concatenate: {
        need(op.axis >= 0 && op.axis < rr, "concatenate dim");
        int64_t sum = 0;
        for (int o : op.operands) {
          const auto& is = T(o).shape;
          need((int)is.size() == rr, "concatenate rank");
          for (int i = 0; i < rr && (int)is.size() == rr; ++i)
            if (i != op.axis) need(is[i] == rs[i], "concatenate extent");
          if ((int)is.size() == rr) sum += is[op.axis];
        }
        need(sum == rs[op.axis], "concatenate total extent");
        break;
      }
      case OpKind::Reverse:
        need(T(op.operands[0]).shape == rs, "reverse shape");
        for (auto d : op.dims) need(d >= 0 && d < rr, "reverse dim");
        break;
      case OpKind::Reduce: {
        const auto& is = T(op.operands[0]).shape;
        need(T(op.operands[1]).shape.empty(), "reduce init must be a scalar");
        std::vector<int64_t> keep;
        std::vector<int> seen(is.size(), 0);
        for (auto d : op.dims) need(d >= 0 && d < (int64_t)is.size() && !seen[d]++, "reduce dims");
        for (size_t i = 0; i < is.size(); ++i)
          if (!seen[i]) keep.push_back(is[i]);
        need(keep == rs, "reduce result shape");
        break;
      }
      case OpKind::DotGeneral: {
        const auto& a = T(op.operands[0]).shape;
        const auto& b = T(op.operands[1]).shape;
        need(op.lb.size() == op.rb.size() && op.lc.size() == op.rc.size(), "dot_general dim arity");
        std::vector<int> ua(a.size(), 0), ub(b.size(), 0);
        std::vector<int64_t> res;
        for (size_t i = 0; i < op.lb.size(); ++i) {
          need(op.lb[i] >= 0 && op.lb[i] < (int64_t)a.size() && op.rb[i] >= 0 && op.rb[i] < (int64_t)b.size(),
               "dot_general batch dim");
          need(!ua[op.lb[i]]++ && !ub[op.rb[i]]++, "dot_general repeated dim");
          need(a[op.lb[i]] == b[op.rb[i]], "dot_general batch extent");
          res.push_back(a[op.lb[i]]);
        }
        for (size_t i = 0; i < op.lc.size(); ++i) {
          need(op.lc[i] >= 0 && op.lc[i] < (int64_t)a.size() && op.rc[i] >= 0 && op.rc[i] < (int64_t)b.size(),
               "dot_general contracting dim");
          need(!ua[op.lc[i]]++ && !ub[op.rc[i]]++, "dot_general repeated dim");
          need(a[op.lc[i]] == b[op.rc[i]], "dot_general contracting extent");
        }
        for (size_t i = 0; i < a.size(); ++i) if (!ua[i]) res.push_back(a[i]);
        for (size_t i = 0; i < b.size(); ++i) if (!ub[i]) res.push_back(b[i]);
        need(res == rs, "dot_general result shape");
        need(T(op.operands[0]).dtype == T(op.operands[1]).dtype &&
                 (T(op.operands[0]).dtype == DType::F32 || T(op.operands[0]).dtype == DType::BF16) &&
                 op.type.dtype == DType::F32,
             "dot_general supports f32 x f32 or bf16 x bf16 operands with an f32 result");
        break;
      }
      case OpKind::Gather: {
        const auto& t = T(op.operands[0]).shape;
        const auto& ix = T(op.operands[1]).shape;
        need(op.slice_sizes.size() == t.size(), "gather slice_sizes arity");
        for (size_t d = 0; d < t.size(); ++d) need(op.slice_sizes[d] >= 0 && op.slice_sizes[d] <= t[d], "gather slice size");
        for (auto d : op.collapsed) need(d >= 0 && d < (int64_t)t.size() && op.slice_sizes[d] <= 1, "gather collapsed dim");
        for (auto d : op.start_index_map) need(d >= 0 && d < (int64_t)t.size(), "gather start_index_map");
        need(op.axis >= 0 && op.axis <= (int64_t)ix.size(), "gather index_vector_dim");
        int64_t nvec = op.axis < (int64_t)ix.size() ? ix[op.axis] : 1;
        need(nvec == (int64_t)op.start_index_map.size(), "gather index vector length");
        int64_t batch_rank = (int64_t)ix.size() - (op.axis < (int64_t)ix.size() ? 1 : 0);
        need((int64_t)rs.size() == batch_rank + (int64_t)op.offset_dims.size(), "gather result rank");
        need(op.offset_dims.size() + op.collapsed.size() == t.size(), "gather offset dims");
        for (auto d : op.offset_dims) need(d >= 0 && d < rr, "gather offset dim");
        std::vector<int64_t> offs_sizes;
        for (size_t d = 0; d < t.size(); ++d)
          if (!std::count(op.collapsed.begin(), op.collapsed.end(), (int64_t)d)) offs_sizes.push_back(op.slice_sizes[d]);
        for (size_t k = 0; k < op.offset_dims.size() && k < offs_sizes.size(); ++k)
          if (op.offset_dims[k] >= 0 && op.offset_dims[k] < rr) need(rs[op.offset_dims[k]] == offs_sizes[k], "gather offset extent");
        break;
      }
      case OpKind::AttnFwd: case OpKind::AttnBwd: {
        const size_t arity = op.kind == OpKind::AttnFwd ? 3 : 6;
        need(op.operands.size() == arity, "attention arity");
        if (op.operands.size() != arity) break;
        const auto& q = T(op.operands[0]).shape;
        need(q.size() == 4 && q[3] == 64, "attention operand shape");
        if (q.size() != 4) break;
        const std::vector<int64_t> rows{q[0], q[1], q[2]};
        const int n4 = op.kind == OpKind::AttnFwd ? 3 : 5;
        for (size_t s = 0; s < op.operands.size(); ++s) {
          need(T(op.operands[s]).dtype == DType::F32, "attention operands are f32");
          need(T(op.operands[s]).shape == ((int)s < n4 ? q : rows), "attention operand shape");
        }
        const int64_t N = q[0] * q[1] * q[2] * 64, R = q[0] * q[1] * q[2];
        need(rs == std::vector<int64_t>{op.kind == OpKind::AttnBwd ? 3 * N + R : N + R}, "attention result size");
        break;
      }
      default:
        break;
    }
  }
  for (size_t j = 0; j < f.returns.size(); ++j)
    if (!(f.value_types[f.returns[j]] == f.results[j]))
      throw std::runtime_error("return value " + std::to_string(j) + " does not match the declared result type");
}

// Every address a GEMM operand view touches must lie inside its base buffer.
void check_view_bounds(const Function& f, const View& v, const char* what) {
  int64_t lo = v.offset, hi = v.offset;
  for (size_t i = 0; i < v.shape.size(); ++i) {
    if (v.shape[i] == 0) return;
    int64_t span = (v.shape[i] - 1) * v.strides[i];
    if (span > 0) hi += span;
    else lo += span;
  }
  int64_t n = f.value_types[v.value].numel();
  if (lo < 0 || hi >= n)
    throw std::runtime_error(std::string("internal: ") + what + " view exceeds its buffer");
}

}  // namespace

namespace {

// True when g is Sheaf's gelu of h, element by element: g's cone back to h
// holds only element-wise ops and splat constants (no index maps), and its
// value at sample points equals 0.5 x (1 + tanh(0.7978846 (x + 0.044715
// x^3))) (sheaf/lib/nn.shf) to 1e-6.  The GEMM epilogue computes exactly
// that form, so fusing it cannot change what is computed beyond rounding.
bool is_gelu_of(const Function& f, int g, int h) {
  if (f.value_types[g].dtype != DType::F32 || f.value_types[h].dtype != DType::F32 ||
      f.value_types[g].shape != f.value_types[h].shape)
    return false;
  std::function<bool(int, double, double*)> eval = [&](int v, double x, double* out) -> bool {
    if (v == h) {
      *out = x;
      return true;
    }
    const int pi = f.producer[v];
    if (pi < 0) return false;
    const Op& op = f.ops[pi];
    if (op.kind == OpKind::Constant) {
      if (op.values.size() != 1) return false;
      *out = op.values[0];
      return true;
    }
    if (op.kind == OpKind::BroadcastInDim) {
      const int src = op.operands[0];
      if (f.value_types[src].numel() != 1) return false;  // splat constants only
      return eval(src, x, out);
    }
    if (f.value_types[v].shape != f.value_types[g].shape && f.value_types[v].numel() != 1) return false;
    double a = 0, b = 0;
    if (is_unary_elementwise(op.kind)) {
      if (!eval(op.operands[0], x, &a)) return false;
      switch (op.kind) {
        case OpKind::Tanh: *out = std::tanh(a); return true;
        case OpKind::Exp: *out = std::exp(a); return true;
        case OpKind::Neg: *out = -a; return true;
        case OpKind::Logistic: *out = 1.0 / (1.0 + std::exp(-a)); return true;
        default: return false;
      }
    }
    if (is_binary_elementwise(op.kind)) {
      if (!eval(op.operands[0], x, &a) || !eval(op.operands[1], x, &b)) return false;
      switch (op.kind) {
        case OpKind::Add: *out = a + b; return true;
        case OpKind::Sub: *out = a - b; return true;
        case OpKind::Mul: *out = a * b; return true;
        case OpKind::Div: *out = a / b; return true;
        case OpKind::Pow: *out = std::pow(a, b); return true;
        default: return false;
      }
    }
    return false;
  };
  for (double x : {-4.5, -2.2, -1.0, -0.37, 0.0, 0.21, 0.8, 1.6, 3.3, 6.0}) {
    double got = 0;
    if (!eval(g, x, &got)) return false;
    const double ref = 0.5 * x * (1.0 + std::tanh(0.7978846 * (x + 0.044715 * x * x * x)));
    if (!(std::fabs(got - ref) <= 1e-6 * (1.0 + std::fabs(ref)))) return false;
  }
  return true;
}

// Fuses a loop step that computes only gelu of a GEMM step's result into the
// GEMM's epilogue: the GEMM writes both h and gelu(h), and the loop step and
// its launch (a read of h) are gone.  h keeps its own consumers (the gelu
// VJP reads it).  Tensor-core modes only: in fp32 mode the GEMM runs on CUDA
// cores and the epilogue would run as its separate unfused kernel anyway.
void fuse_gemm_epilogues(const Function& f, Plan& plan, const std::vector<int>& round_roots,
                         const std::set<int>& consts, std::map<int, int>& step_of_value) {
  std::vector<char> drop(plan.steps.size(), 0);
  std::map<int, int> gemm_step;  // GEMM result -> step
  for (int si = 0; si < (int)plan.steps.size(); ++si) {
    Step& st = plan.steps[si];
    if (st.kind == StepKind::Gemm && st.gemm.epi == 0 && st.extra_roots.empty()) gemm_step[st.root] = si;
    if (st.kind != StepKind::Loop || !st.finish_kernel.empty() || !st.extra_roots.empty() || st.scratch_elems ||
        !st.shadow_values.empty())
      continue;
    int h = -1;
    bool ok = true;
    for (int l : st.leaves) {
      if (consts.count(l)) continue;
      if (h >= 0 && h != l) ok = false;
      h = l;
    }
    if (!ok || h < 0) continue;
    auto it = gemm_step.find(h);
    if (it == gemm_step.end() || !is_gelu_of(f, st.root, h)) continue;
    Step& gs = plan.steps[it->second];
    gs.gemm.epi = kEpiGelu;
    gs.gemm.round_out2 = std::find(round_roots.begin(), round_roots.end(), st.root) != round_roots.end();
    gs.extra_roots.push_back(st.root);
    gs.bytes_moved += st.elements * 4;
    gemm_step.erase(it);
    drop[si] = 1;
  }
  if (std::find(drop.begin(), drop.end(), 1) == drop.end()) return;
  std::vector<Step> kept;
  std::vector<int> new_index(plan.steps.size(), -1);
  for (size_t si = 0; si < plan.steps.size(); ++si) {
    if (drop[si]) continue;
    new_index[si] = (int)kept.size();
    kept.push_back(std::move(plan.steps[si]));
  }
  plan.steps = std::move(kept);
  for (auto& [v, si] : step_of_value) {
    if (new_index[si] >= 0) {
      si = new_index[si];
      continue;
    }
    // a fused loop's root: written by its GEMM step now
    for (int k = 0; k < (int)plan.steps.size(); ++k)
      for (int e : plan.steps[k].extra_roots)
        if (e == v) si = k;
  }
}

Plan plan_function(const Function& f, Precision prec) {
  verify(f);
  Planner pl(f, prec);
  pl.liveness();
  for (int iter = 0;; ++iter) {
    if (iter > 64) throw std::runtime_error("planner did not converge");
    pl.clusterize();
    if (pl.validate_remat()) continue;
    bool retry = pl.absorb_reduce_epilogues();
    for (size_t i = 0; i < f.ops.size(); ++i) {
      const Op& op = f.ops[i];
      if (!pl.live[op.result]) continue;
      if (pl.is_gemm_root(op)) {
        GemmDesc g;
        if (!pl.gemm_of(op, &g)) retry = true;
      } else if (is_attention(op.kind)) {
        AttnDesc d;
        if (!pl.attn_of(op, &d)) retry = true;
      } else if (op.kind == OpKind::Gather) {
        View t;
        if (!pl.view_of(op.operands[0], &t)) {
          pl.forced.insert(op.operands[0]);
          retry = true;
        }
      }
    }
    if (!retry) break;
  }

  Plan plan;
  plan.fn = &f;
  int NV = pl.NV;
  plan.value_offset.assign(NV, -1);
  for (size_t i = 0; i < f.ops.size(); ++i) {
    const Op& op = f.ops[i];
    if (pl.live[op.result] && pl.cluster[op.result] == kConst) plan.constants.push_back(op.result);
  }

  // TF32: operands are rounded to nearest TF32 where they are produced (the
  // tensor cores would truncate them).  Parameters read by GEMMs get rounded
  // copies; step roots consumed only by GEMMs and attention are stored rounded
  // (GEMM and attention steps in their epilogues, loops as they store).
  std::set<int> round_gemm_outputs;
  std::vector<int> round_roots;
  std::map<int, int> shadow_of;  // value -> index into plan.shadows
  if (prec == Precision::TF32 || prec == Precision::BF16) {
    std::set<int> bases, attn_bases;
    for (const Op& op : f.ops) {
      if (!pl.live[op.result]) continue;
      if (is_attention(op.kind)) {
        AttnDesc d;
        if (pl.attn_of(op, &d))
          for (const View& w : d.in)
            if (w.shape.size() == 4) attn_bases.insert(w.value);
        continue;
      }
      if (!pl.is_gemm_root(op)) continue;
      GemmDesc g;
      // skinny GEMMs (at most kSkinnyMax rows or columns) run in f32 on the
      // CUDA cores: their operands need no TF32 rounding or bf16 copy
      if (pl.gemm_of(op, &g) && g.M > kSkinnyMax && g.N > kSkinnyMax) {
        bases.insert(g.a.value);
        bases.insert(g.b.value);
      }
    }
    const std::set<int> gemm_bases = bases;
    if (prec == Precision::BF16) {
      // bf16 contractions: every f32 GEMM operand (parameter or step result)
      // is read through a bf16 shadow; attention keeps TF32 operands
      bases.clear();
      for (int v : gemm_bases) {
        if (f.value_types[v].dtype != DType::F32) continue;
        if (pl.cluster[v] != kParam && pl.cluster[v] != v) continue;
        Shadow sh;
        sh.value = v;
        sh.dtype = DType::BF16;
        shadow_of[v] = (int)plan.shadows.size();
        plan.shadows.push_back(sh);
      }
    }
    bases.insert(attn_bases.begin(), attn_bases.end());
    for (int v : bases) {
      if (pl.cluster[v] == kParam && f.value_types[v].dtype == DType::F32) {
        plan.rounded_params.push_back(v);
      } else if (pl.cluster[v] == v && pl.only_gemm_consumers(v)) {
        const Op* p = pl.producer(v);
        if (p && (pl.is_gemm_root(*p) || is_attention(p->kind))) round_gemm_outputs.insert(v);
        else round_roots.push_back(v);
      } else if (prec == Precision::TF32 && pl.cluster[v] == v && gemm_bases.count(v) &&
                 f.value_types[v].dtype == DType::F32) {
        // read by GEMMs and by other steps (e.g. the residual-stream gradient,
        // which feeds a projection's backward GEMMs and the next residual
        // add): the GEMMs read a rounded shadow copy.  Unrounded, the tensor
        // cores would truncate it -- a one-sided error that does not average
        // out over the contraction.
        Shadow sh;
        sh.value = v;
        shadow_of[v] = (int)plan.shadows.size();
        plan.shadows.push_back(sh);
      }
    }
  }
  CodeGen cg(f, pl.cluster);
  cg.set_round_roots(round_roots);
  {
    // shadows of step results: written by the producing row-group kernel
    // where it can (Step::shadow_values), else by a conversion step
    std::map<int, DType> sv;
    for (const Shadow& sh : plan.shadows)
      if (pl.cluster[sh.value] != kParam) sv[sh.value] = sh.dtype;
    cg.set_shadow_values(sv);
  }
  std::map<int, int> step_of_value;
  // Consecutive loop / row-reduction steps over the same rows run as one row
  // group (CodeGen::gen_row_group): one launch, and each row's intermediates
  // are re-read from L1/L2 by the warp that just wrote them.
  struct Member {
    CodeGen::RowMember m;
    int op_index, value;
  };
  std::vector<Member> group;
  std::map<int, int> inside;  // member output -> 0 ([rows..., C]) or 1 (row)
  int64_t gR = 0, gC = 0;
  // SHEAF_B200_ROW_GROUPS=0 plans every step as its own kernel (for comparison)
  const char* rg_env = std::getenv("SHEAF_B200_ROW_GROUPS");
  const bool row_groups = !(rg_env && std::string(rg_env) == "0");
  auto emit_single = [&](size_t i) {
    const Op& op = f.ops[i];
    const int v = op.result;
    Step st;
    st.root = v;
    st.elements = op.type.numel();
    st.kind = StepKind::Reduce;
    if (op.kind == OpKind::Reduce) {
      cg.gen_reduce(op, &st);
    } else if (pl.epilogue_of.count(v)) {
      cg.gen_reduce(f.ops[f.producer[pl.epilogue_of[v]]], &st, &op);
    } else {
      st.kind = StepKind::Loop;
      cg.gen_loop(op, &st);
    }
    step_of_value[v] = (int)plan.steps.size();
    plan.materialized.push_back(v);
    plan.steps.push_back(std::move(st));
  };
  // Emits the pending members: the longest run from the first one that the
  // row-group generator accepts (a member it cannot express, e.g. a gather,
  // is emitted as its own kernel), and so on.
  auto flush = [&]() {
    size_t b = 0;
    while (b < group.size()) {
      size_t done = 0;
      for (size_t e = group.size(); e >= b + 2 && !done; --e) {
        std::vector<CodeGen::RowMember> ms;
        for (size_t k = b; k < e; ++k) ms.push_back(group[k].m);
        Step st;
        st.kind = StepKind::Loop;
        if (!cg.gen_row_group(ms, gR, gC, &st)) continue;
        for (size_t k = b; k < e; ++k) {
          step_of_value[group[k].value] = (int)plan.steps.size();
          plan.materialized.push_back(group[k].value);
        }
        plan.steps.push_back(std::move(st));
        done = e - b;
      }
      if (done) {
        b += done;
      } else {
        emit_single((size_t)group[b].op_index);
        ++b;
      }
    }
    group.clear();
    inside.clear();
  };
  // row-group role of the loop / reduction step rooted at op i: kind (-1: none)
  auto row_role = [&](size_t i, int64_t* R, int64_t* C, CodeGen::RowMember* m) {
    const Op& op = f.ops[i];
    const int v = op.result;
    // f32 or bf16 (computed in f32, rounded to bf16 per op as everywhere)
    const bool bf = op.type.dtype == DType::BF16;
    if (op.type.dtype != DType::F32 && !bf) return -1;
    const Op* red = nullptr;
    if (op.kind == OpKind::Reduce) red = &op;
    else if (pl.epilogue_of.count(v)) red = &f.ops[f.producer[pl.epilogue_of[v]]];
    if (red) {
      const auto& is = f.value_types[red->operands[0]].shape;
      // column reduction over every dim but the innermost
      bool col = !bf && red == &op && is.size() >= 2 && red->dims.size() == is.size() - 1 &&
                 f.value_types[red->operands[0]].dtype == DType::F32;
      for (size_t d = 0; col && d + 1 < is.size(); ++d) col = red->dims[d] == (int64_t)d;
      if (col) {
        *C = is.back();
        *R = f.value_types[red->operands[0]].numel() / std::max<int64_t>(*C, 1);
        *m = {3, red, nullptr};
        return 3;
      }
      const DType idt = f.value_types[red->operands[0]].dtype;
      if (red->dims.size() != 1 || is.empty() || red->dims[0] != (int64_t)is.size() - 1 ||
          (idt != DType::F32 && idt != DType::BF16))
        return -1;
      *R = red->type.numel();
      *C = is.back();
      *m = {2, red, red == &op ? nullptr : &op};
      return 2;
    }
    const auto& sh = op.type.shape;
    if (sh.empty()) return -1;
    *R = op.type.numel() / std::max<int64_t>(sh.back(), 1);
    *C = sh.back();
    *m = {0, &op, nullptr};
    return 0;
  };
  for (size_t i = 0; i < f.ops.size(); ++i) {
    const Op& op = f.ops[i];
    int v = op.result;
    if (!pl.live[v] || pl.cluster[v] != v) continue;
    const bool generated = !(pl.is_gemm_root(op) || is_attention(op.kind) || op.kind == OpKind::SortPairs ||
                             op.kind == OpKind::ScatterAddRows);
    if (generated) {
      int64_t R = 0, C = 0;
      CodeGen::RowMember m{};
      int kind = row_role(i, &R, &C, &m);
      const int member_root = m.epi ? m.epi->result : (m.root ? m.root->result : -1);
      if (!group.empty() && kind == 0 && op.type.numel() == gR && R * C == gR) {
        kind = 1;  // a loop over the group's rows
        m.kind = 1;
        R = gR;
        C = gC;
      }
      if (!row_groups) kind = -1;
      const bool fits = kind >= 0 && R == gR && C == gC && !group.empty();
      std::set<std::pair<int, int>> seen;
      // class of the member's output inside the group: 0 per element, 1 per
      // row, 2 not readable by later members (a column reduction)
      const int cls = kind == 0 ? 0 : kind == 3 ? 2 : 1;
      if (fits && pl.row_local(member_root, cls, member_root, inside, gR, gC, seen)) {
        group.push_back({m, (int)i, v});
        inside[v] = cls;
        continue;
      }
      flush();
      if (kind == 0 || kind == 2 || kind == 3) {
        if (R >= 1024 && C >= 32 && C <= 2048) {
          gR = R;
          gC = C;
          group.push_back({m, (int)i, v});
          inside[v] = cls;
          continue;
        }
      }
      emit_single(i);
      continue;
    }
    flush();
    Step st;
    st.root = v;
    st.elements = op.type.numel();
    if (pl.is_gemm_root(op)) {
      st.kind = StepKind::Gemm;
      if (!pl.gemm_of(op, &st.gemm)) fail(op, "internal: GEMM operand views changed after planning");
      st.gemm.round_out = round_gemm_outputs.count(v) > 0;
      for (int rp : plan.rounded_params) {
        if (st.gemm.a.value == rp) st.gemm.a_rounded = true;
        if (st.gemm.b.value == rp) st.gemm.b_rounded = true;
      }
      {
        const int sa = shadow_of.count(st.gemm.a.value) ? shadow_of[st.gemm.a.value] : -1;
        const int sb = shadow_of.count(st.gemm.b.value) ? shadow_of[st.gemm.b.value] : -1;
        const bool bf_a = sa >= 0 && plan.shadows[sa].dtype == DType::BF16;
        const bool bf_b = sb >= 0 && plan.shadows[sb].dtype == DType::BF16;
        if (bf_a == bf_b) {  // bf16 shadows only in pairs: both operands or neither
          st.gemm.a_shadow = sa;
          st.gemm.b_shadow = sb;
        } else {
          st.gemm.a_shadow = bf_a ? -1 : sa;
          st.gemm.b_shadow = bf_b ? -1 : sb;
        }
        st.gemm.bf16 = (bf_a && bf_b) || f.value_types[st.gemm.a.value].dtype == DType::BF16;
      }
      check_view_bounds(f, st.gemm.a, "GEMM lhs");
      check_view_bounds(f, st.gemm.b, "GEMM rhs");
      st.leaves = {st.gemm.a.value, st.gemm.b.value};
      st.flops = 2.0 * st.gemm.batch * st.gemm.M * st.gemm.N * st.gemm.K;
      {
        const int64_t es = st.gemm.bf16 ? 2 : 4;  // operand bytes; C is f32
        st.bytes_moved = st.gemm.batch * (es * (st.gemm.M * st.gemm.K + st.gemm.K * st.gemm.N) + 4 * st.gemm.M * st.gemm.N);
      }
    } else if (is_attention(op.kind)) {
      st.kind = StepKind::Attn;
      if (!pl.attn_of(op, &st.attn)) fail(op, "internal: attention operand views changed after planning");
      st.attn.round_out = round_gemm_outputs.count(v) > 0 || (prec == Precision::TF32 && pl.only_gemm_consumers(v));
      for (const View& w : st.attn.in) {
        check_view_bounds(f, w, "attention operand");
        st.leaves.push_back(w.value);
        st.attn.rounded.push_back(w.shape.size() == 4 && std::count(plan.rounded_params.begin(),
                                                                     plan.rounded_params.end(), w.value) > 0);
      }
      const AttnDesc& a = st.attn;
      const double T = (double)a.T, pairs = a.causal ? T * (T + 1) / 2 : T * T;
      const double prod = 2.0 * a.B * a.H * 64 * pairs;  // one T x T x 64 product
      const int64_t N = a.B * a.H * a.T * 64, R = a.B * a.H * a.T;
      if (op.kind == OpKind::AttnFwd) {
        st.flops = 2 * prod;
        st.bytes_moved = 4 * (3 * N + N + R);
      } else {
        // dQ pass (3 products): q, k, v, dY, Y, L in, dQ, D out; dK/dV pass
        // (4 products): q, k, v, dY, L, D in, dK, dV out
        st.flops = 7 * prod;
        st.bytes_moved = 4 * ((5 * N + R + N + R) + (4 * N + 2 * R + 2 * N));
      }
    } else if (op.kind == OpKind::ScatterAddRows) {
      st.kind = StepKind::Scatter;
      for (int o : op.operands)
        if (!pl.materialized(o)) fail(op, "internal: scatter operand is not materialized");
      st.leaves = {op.operands[0], op.operands[1]};
      const int64_t n = f.value_types[op.operands[0]].numel(), V = op.type.shape[0], D = op.type.shape[1];
      st.gemm.M = V;
      st.gemm.N = D;
      st.gemm.K = n;
      // workspace (ints) for the counting sort, in the step's scratch
      st.scratch_elems = ((int64_t)scatter_add_rows_workspace(n, V, D) + 3) / 4;
      st.splits = 1;
      st.bytes_moved = 4 * (n + n * D + V * D);
    } else if (op.kind == OpKind::SortPairs) {
      // operands are materialized dense buffers (a sort consumer blocks fusion)
      st.kind = StepKind::Sort;
      for (int o : op.operands)
        if (!pl.materialized(o)) fail(op, "internal: sort operand is not materialized");
      st.leaves = {op.operands[0], op.operands[1]};
      const int64_t n = f.value_types[op.operands[0]].shape.back();
      st.gemm.M = f.value_types[op.operands[0]].numel() / std::max<int64_t>(n, 1);  // rows
      st.gemm.N = n;
      st.gemm.K = op.axis;  // 1: descending
      st.bytes_moved = 16 * f.value_types[op.operands[0]].numel();
    }
    step_of_value[v] = (int)plan.steps.size();
    plan.materialized.push_back(v);
    plan.steps.push_back(std::move(st));
  }
  flush();
  if (prec == Precision::TF32 || prec == Precision::BF16) {
    std::set<int> consts(plan.constants.begin(), plan.constants.end());
    fuse_gemm_epilogues(f, plan, round_roots, consts, step_of_value);
  }
  // conversion steps of the operand shadows, each right after the step that
  // writes its value
  if (!plan.shadows.empty()) {
    // drop shadows no GEMM reads (a bf16 shadow whose partner operand has none)
    {
      std::vector<char> used(plan.shadows.size(), 0);
      for (const Step& st0 : plan.steps) {
        if (st0.kind == StepKind::Gemm)
          for (int k : {st0.gemm.a_shadow, st0.gemm.b_shadow})
            if (k >= 0) used[k] = 1;
        // a shadow a kernel writes keeps its buffer even if no GEMM reads it
        for (int v : st0.shadow_values) used[shadow_of.at(v)] = 1;
      }
      std::vector<int> remap(plan.shadows.size(), -1);
      std::vector<Shadow> kept;
      shadow_of.clear();
      for (size_t k = 0; k < plan.shadows.size(); ++k)
        if (used[k]) {
          remap[k] = (int)kept.size();
          shadow_of[plan.shadows[k].value] = (int)kept.size();
          kept.push_back(plan.shadows[k]);
        }
      plan.shadows = std::move(kept);
      for (Step& st0 : plan.steps)
        if (st0.kind == StepKind::Gemm) {
          if (st0.gemm.a_shadow >= 0) st0.gemm.a_shadow = remap[st0.gemm.a_shadow];
          if (st0.gemm.b_shadow >= 0) st0.gemm.b_shadow = remap[st0.gemm.b_shadow];
        }
    }
    std::vector<Step> steps;
    std::vector<int> new_index(plan.steps.size(), -1);
    // shadows of parameters: converted first, once per call
    for (size_t k = 0; k < plan.shadows.size(); ++k) {
      Shadow& sh = plan.shadows[k];
      if (pl.cluster[sh.value] != kParam) continue;
      Step cs;
      cs.kind = StepKind::Convert;
      cs.root = sh.value;
      cs.leaves = {sh.value};
      cs.shadow = (int)k;
      cs.elements = f.value_types[sh.value].numel();
      cs.bytes_moved = cs.elements * (4 + dtype_bytes(sh.dtype));
      sh.step = (int)steps.size();
      steps.push_back(std::move(cs));
    }
    for (size_t si = 0; si < plan.steps.size(); ++si) {
      Step& st0 = plan.steps[si];
      std::vector<int> written{st0.root};
      written.insert(written.end(), st0.extra_roots.begin(), st0.extra_roots.end());
      new_index[si] = (int)steps.size();
      for (int v : st0.shadow_values) {
        const int k = shadow_of.at(v);
        st0.shadow_outs.push_back(k);
        plan.shadows[k].step = (int)steps.size();
      }
      const std::vector<int> fused = st0.shadow_values;
      steps.push_back(std::move(st0));
      for (int w : written) {
        auto it = shadow_of.find(w);
        if (it == shadow_of.end()) continue;
        if (std::find(fused.begin(), fused.end(), w) != fused.end()) continue;  // written by the kernel
        Shadow& sh = plan.shadows[it->second];
        Step cs;
        cs.kind = StepKind::Convert;
        cs.root = w;
        cs.leaves = {w};
        cs.shadow = it->second;
        cs.elements = f.value_types[w].numel();
        cs.bytes_moved = cs.elements * (4 + dtype_bytes(sh.dtype));
        sh.step = (int)steps.size();
        steps.push_back(std::move(cs));
      }
    }
    plan.steps = std::move(steps);
    for (auto& [v, si] : step_of_value) si = new_index[si];
    for (int si = 0; si < (int)plan.steps.size(); ++si) {
      const Step& st0 = plan.steps[si];
      if (st0.kind != StepKind::Gemm) continue;
      for (int k : {st0.gemm.a_shadow, st0.gemm.b_shadow})
        if (k >= 0) plan.shadows[k].last_use = std::max(plan.shadows[k].last_use, si);
    }
    for (const Shadow& sh : plan.shadows)
      if (sh.step < 0)
        throw std::runtime_error("internal: operand shadow of %" + std::to_string(sh.value) +
                                 " without a producing step");
  }
  plan.source = cg.source();
  plan.snippets = cg.snippets();
  plan.prelude = CodeGen::prelude();
  plan.kernel_names = cg.kernel_names();

  // Output slots: first occurrence of a step root writes the output buffer directly.
  plan.output_step.assign(f.returns.size(), -1);
  {
    std::set<int> seen;
    for (size_t j = 0; j < f.returns.size(); ++j) {
      int v = f.returns[j];
      if (pl.cluster[v] == v && !seen.count(v)) {
        plan.output_step[j] = step_of_value[v];
        seen.insert(v);
      }
    }
  }

  // Arena: intermediates that are not outputs, plus split-reduction scratch.
  struct Interval { int64_t bytes; int start, end; int value; int step_scratch; };
  std::vector<Interval> iv;
  std::vector<int> last_use(NV, -1);
  for (int s = 0; s < (int)plan.steps.size(); ++s)
    for (int l : plan.steps[s].leaves) last_use[l] = std::max(last_use[l], s);
  // a row group's column sums whose outputs no later step reads may be
  // finished at the end of the call (batched): their partials live until then
  for (int s = 0; s < (int)plan.steps.size(); ++s) {
    Step& st = plan.steps[s];
    if (st.col_finish.empty()) continue;
    bool read_later = false;
    for (const Step::ColFinish& cf : st.col_finish) {
      const int v = cf.out == 0 ? st.root : st.extra_roots[cf.out - 1];
      read_later = read_later || last_use[v] > s;
    }
    st.finish_deferred = !read_later;
  }
  for (int s = 0; s < (int)plan.steps.size(); ++s) {
    // a conversion step writes a shadow (placed below), not its root value
    if (plan.steps[s].kind == StepKind::Convert) continue;
    std::vector<int> written{plan.steps[s].root};
    written.insert(written.end(), plan.steps[s].extra_roots.begin(), plan.steps[s].extra_roots.end());
    for (int v : written) {
      if (pl.returned[v]) continue;
      int64_t bytes = f.value_types[v].numel() * dtype_bytes(f.value_types[v].dtype);
      iv.push_back({bytes, s, std::max(s, last_use[v]), v, -1});
    }
    const int scratch_end = plan.steps[s].finish_deferred ? (int)plan.steps.size() - 1 : s;
    if (plan.steps[s].scratch_elems && !pl.returned[plan.steps[s].root])
      iv.push_back({plan.steps[s].scratch_elems * 4, s, scratch_end, -1, s});
  }
  for (int s = 0; s < (int)plan.steps.size(); ++s)
    if (plan.steps[s].scratch_elems && pl.returned[plan.steps[s].root])
      iv.push_back({plan.steps[s].scratch_elems * 4, s,
                    plan.steps[s].finish_deferred ? (int)plan.steps.size() - 1 : s, -1, s});
  int last_gemm = -1;
  for (int s2 = 0; s2 < (int)plan.steps.size(); ++s2)
    if (plan.steps[s2].kind == StepKind::Gemm || plan.steps[s2].kind == StepKind::Attn) last_gemm = s2;
  for (int rp : plan.rounded_params)
    iv.push_back({f.value_types[rp].numel() * 4, 0, std::max(last_gemm, 0), -1, -2 - rp});
  // operand shadows: step_scratch encodes -(2 + NV + shadow index)
  for (size_t k = 0; k < plan.shadows.size(); ++k) {
    const Shadow& sh = plan.shadows[k];
    iv.push_back({f.value_types[sh.value].numel() * dtype_bytes(sh.dtype), sh.step, std::max(sh.step, sh.last_use), -1,
                  -2 - NV - (int)k});
  }
  std::vector<int> order(iv.size());
  for (size_t i = 0; i < iv.size(); ++i) order[i] = (int)i;
  std::sort(order.begin(), order.end(), [&](int x, int y) { return iv[x].bytes > iv[y].bytes; });
  std::vector<std::pair<int64_t, int>> placed;  // offset, interval
  std::vector<int64_t> off(iv.size(), 0);
  int64_t total = 0;
  auto align = [](int64_t x) { return (x + 255) & ~int64_t(255); };
  for (int k : order) {
    std::vector<std::pair<int64_t, int64_t>> busy;
    for (auto& [o, j] : placed)
      if (!(iv[j].end < iv[k].start || iv[k].end < iv[j].start)) busy.push_back({o, o + align(iv[j].bytes)});
    std::sort(busy.begin(), busy.end());
    int64_t cand = 0;
    for (auto& [b, e] : busy) {
      if (cand + align(iv[k].bytes) <= b) break;
      cand = std::max(cand, e);
    }
    off[k] = cand;
    placed.push_back({cand, k});
    total = std::max(total, cand + align(iv[k].bytes));
  }
  plan.scratch_offset.assign(plan.steps.size(), -1);
  plan.rounded_offset.assign(plan.rounded_params.size(), -1);
  for (size_t k = 0; k < iv.size(); ++k) {
    if (iv[k].value >= 0) plan.value_offset[iv[k].value] = off[k];
    else if (iv[k].step_scratch >= 0) plan.scratch_offset[iv[k].step_scratch] = off[k];
    else if (-2 - iv[k].step_scratch >= NV) {
      plan.shadows[-2 - NV - iv[k].step_scratch].offset = off[k];
    } else {
      int rp = -2 - iv[k].step_scratch;
      for (size_t j = 0; j < plan.rounded_params.size(); ++j)
        if (plan.rounded_params[j] == rp) plan.rounded_offset[j] = off[k];
    }
  }
  plan.arena_bytes = total;
  return plan;
}

}  // namespace

namespace {

bool is_identity_init(const Function& f, int v, ReduceBody body) {
  const int pi = f.producer[v];
  if (pi < 0) return false;
  const Op& op = f.ops[pi];
  if (op.kind != OpKind::Constant || op.values.size() != 1) return false;
  const double x = op.values[0];
  switch (body) {
    case ReduceBody::Add: return x == 0.0;
    case ReduceBody::Mul: return x == 1.0;
    case ReduceBody::Max: return std::isinf(x) && x < 0;
    case ReduceBody::Min: return std::isinf(x) && x > 0;
  }
  return false;
}

// reduce(reduce(x, D1), D2) with one body, identity inits and a single-use
// inner value -> reduce(x, D1 + D2 mapped to x's dims).  Sheaf's sum_to_shape
// emits such chains (one single-axis reduce per broadcast axis, e.g. the
// [B,T,D] -> [D] gradient of a layer-norm gain); merged, the sum is one pass.
// Reductions of a dot_general are left alone (they fold into the GEMM).
std::unique_ptr<Function> merge_reduce_chains(const Function& f) {
  std::vector<int> uses(f.num_values(), 0);
  std::vector<char> returned(f.num_values(), 0);
  for (int r : f.returns) returned[r] = 1;
  for (const Op& op : f.ops)
    for (int o : op.operands) ++uses[o];
  std::unique_ptr<Function> g;
  for (size_t i = 0; i < f.ops.size(); ++i) {
    const Function& cur = g ? *g : f;
    const Op& r2 = cur.ops[i];
    if (r2.kind != OpKind::Reduce) continue;
    const int v = r2.operands[0];
    const int pi = cur.producer[v];
    if (pi < 0 || returned[v] || uses[v] != 1) continue;
    const Op& r1 = cur.ops[pi];
    if (r1.kind != OpKind::Reduce || r1.body != r2.body) continue;
    const int x = r1.operands[0];
    if (cur.producer[x] >= 0 && cur.ops[cur.producer[x]].kind == OpKind::DotGeneral) continue;
    if (!is_identity_init(cur, r1.operands[1], r1.body) || !is_identity_init(cur, r2.operands[1], r2.body)) continue;
    const int rx = (int)cur.value_types[x].shape.size();
    // only chains whose first step keeps the innermost dimension (column
    // reductions: the intermediate is large); a row reduction followed by a
    // small second step is better left as two kernels, which keep per-row
    // terms out of the inner loop
    if (std::count(r1.dims.begin(), r1.dims.end(), (int64_t)(rx - 1))) continue;
    std::vector<int64_t> kept;
    for (int d = 0; d < rx; ++d)
      if (!std::count(r1.dims.begin(), r1.dims.end(), (int64_t)d)) kept.push_back(d);
    std::vector<int64_t> dims(r1.dims.begin(), r1.dims.end());
    bool ok = true;
    for (int64_t d : r2.dims) {
      if (d < 0 || d >= (int64_t)kept.size()) { ok = false; break; }
      dims.push_back(kept[d]);
    }
    if (!ok) continue;
    std::sort(dims.begin(), dims.end());
    if (!g) g = std::make_unique<Function>(f);
    Op merged = g->ops[i];
    merged.operands = {x, r2.operands[1]};
    merged.dims = dims;
    g->ops[i] = merged;
    --uses[v];
    ++uses[x];
  }
  return g;
}

// transpose(dot(L, R)) -> dot(R, L), and transpose(reduce_add over the
// leading batch dim of dot(L, R)) -> reduce_add(dot(R, L)), when the dot (and
// the reduction) have no other use and each operand has one free dim: the
// GEMM writes the transposed layout itself.  Sheaf's weight gradients arrive
// this way (dW = tr(sum_b x_b^T @ g_b)); without the rewrite the GEMM output
// is copied through a transposing loop.
std::unique_ptr<Function> transpose_dot_outputs(const Function& f) {
  std::vector<int> uses(f.num_values(), 0);
  std::vector<char> returned(f.num_values(), 0);
  for (int r : f.returns) returned[r] = 1;
  for (const Op& op : f.ops)
    for (int o : op.operands) ++uses[o];
  auto single = [&](int v) { return v >= 0 && uses[v] == 1 && !returned[v] && f.producer[v] >= 0; };
  // dot with batch dims 0..nb-1 on both sides and one free dim per operand
  auto simple_dot = [&](const Op& d) {
    if (d.kind != OpKind::DotGeneral || d.lb.size() != d.rb.size()) return false;
    const size_t nb = d.lb.size();
    for (size_t i = 0; i < nb; ++i)
      if (d.lb[i] != (int64_t)i || d.rb[i] != (int64_t)i) return false;
    const size_t lr = f.value_types[d.operands[0]].shape.size(), rr = f.value_types[d.operands[1]].shape.size();
    return lr == nb + 1 + d.lc.size() && rr == nb + 1 + d.rc.size() && d.type.shape.size() == nb + 2;
  };
  auto swapped = [](Op d) {
    std::swap(d.operands[0], d.operands[1]);
    std::swap(d.lb, d.rb);
    std::swap(d.lc, d.rc);
    return d;
  };
  std::unique_ptr<Function> g;
  std::vector<char> erase(f.ops.size(), 0);
  for (size_t i = 0; i < f.ops.size(); ++i) {
    const Op& t = f.ops[i];
    if (t.kind != OpKind::Transpose || !single(t.operands[0])) continue;
    const int v = t.operands[0];
    const int pv = f.producer[v];
    const Op& pop = f.ops[pv];
    const size_t r = t.dims.size();
    if (r < 2 || t.dims[r - 1] != (int64_t)r - 2 || t.dims[r - 2] != (int64_t)r - 1) continue;
    bool lead_ident = true;
    for (size_t k = 0; k + 2 < r; ++k) lead_ident = lead_ident && t.dims[k] == (int64_t)k;
    if (!lead_ident) continue;
    if (simple_dot(pop) && pop.lb.size() + 2 == r) {
      if (!g) g = std::make_unique<Function>(f);
      Op d = swapped(pop);
      d.result = t.result;
      d.type = t.type;
      g->ops[pv] = d;
      erase[i] = 1;
      continue;
    }
    // reduce_add over dim 0 of a batched simple dot, 2-D result
    if (pop.kind != OpKind::Reduce || pop.body != ReduceBody::Add || pop.dims.size() != 1 || pop.dims[0] != 0 ||
        r != 2 || !single(pop.operands[0]) || !is_identity_init(f, pop.operands[1], pop.body))
      continue;
    const int dv = pop.operands[0];
    const int pd = f.producer[dv];
    const Op& dop = f.ops[pd];
    if (!simple_dot(dop) || dop.lb.size() != 1) continue;
    if (!g) g = std::make_unique<Function>(f);
    Op d = swapped(dop);
    const auto& ds = f.value_types[dv].shape;
    d.type.shape = {ds[0], ds[2], ds[1]};
    g->value_types[dv] = d.type;
    g->ops[pd] = d;
    Op red = pop;
    red.result = t.result;
    red.type = t.type;
    g->ops[pv] = red;
    erase[i] = 1;
  }
  if (!g) return g;
  std::vector<Op> kept;
  for (size_t i = 0; i < g->ops.size(); ++i)
    if (!erase[i]) kept.push_back(std::move(g->ops[i]));
  g->ops = std::move(kept);
  g->producer.assign(g->num_values(), -1);
  for (size_t i = 0; i < g->ops.size(); ++i) g->producer[g->ops[i].result] = (int)i;
  return g;
}

}  // namespace

Plan build_plan(const Function& f, Precision prec, bool fuse_attention) {
  std::shared_ptr<Function> cur;
  std::string log;
  if ((prec == Precision::TF32 || prec == Precision::BF16) && fuse_attention)
    cur.reset(rewrite_attention(f, &log).release());
  {
    std::string elog;
    if (auto m = rewrite_embedding_grad(cur ? *cur : f, &elog)) {
      cur.reset(m.release());
      log += (log.empty() ? "" : "; ") + elog;
    }
  }
  if (auto m = merge_reduce_chains(cur ? *cur : f)) cur.reset(m.release());
  if (auto m = transpose_dot_outputs(cur ? *cur : f)) cur.reset(m.release());
  std::string mlog;
  if (auto m = merge_sibling_dots(cur ? *cur : f, &mlog)) {
    cur.reset(m.release());
    log += (log.empty() ? "" : "; ") + mlog;
  }
  if (cur) {
    Plan p = plan_function(*cur, prec);
    p.rewritten = cur;
    p.fn = cur.get();
    p.rewrite_log = log;
    return p;
  }
  return plan_function(f, prec);
}

std::string Plan::summary() const {
  std::ostringstream os;
  os.precision(17);
  int loops = 0, reds = 0, gemms = 0, attn = 0, sorts = 0, converts = 0, scatters = 0;
  double flops = 0, aflops = 0;
  for (auto& s : steps) {
    if (s.kind == StepKind::Loop) ++loops;
    else if (s.kind == StepKind::Reduce) ++reds;
    else if (s.kind == StepKind::Attn) { ++attn; aflops += s.flops; continue; }
    else if (s.kind == StepKind::Sort) { ++sorts; continue; }
    else if (s.kind == StepKind::Convert) { ++converts; continue; }
    else if (s.kind == StepKind::Scatter) { ++scatters; continue; }
    else ++gemms;
    flops += s.flops;
  }
  os << "steps=" << steps.size() << " loop=" << loops << " reduce=" << reds << " gemm=" << gemms
     << " attention=" << attn << (sorts ? " sort=" + std::to_string(sorts) : std::string())
     << (converts ? " convert=" + std::to_string(converts) : std::string())
     << (scatters ? " scatter=" + std::to_string(scatters) : std::string()) << " constants=" << constants.size() << " arena_bytes=" << arena_bytes
     << " gemm_flops=" << flops << " attention_flops=" << aflops;
  return os.str();
}

}  // namespace sb
