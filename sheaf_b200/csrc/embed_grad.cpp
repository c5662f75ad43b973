// Embedding-gradient rewrite.
//
// Sheaf's reverse-mode rule for a table lookup `(get table idx)` writes the
// table's adjoint as a product with a transposed one-hot matrix
// (sheaf/src/autodiff/reverse.rs:1015-1041):
//     d_table = transpose(one_hot(idx, V)) @ adj      (summed over batch dims)
// which the emitter lowers to a (batched) dot_general whose left operand is
// the transpose of an element-wise expression of iota and the broadcast index,
// followed, for batched indices, by a reduce over the batch dims (the
// unbroadcast of sum_to_shape).  For a vocabulary of 50304 and 8192 tokens the
// product is 0.63 TFLOP over a 1.65 GB matrix of zeros and ones.  This rewrite
// replaces it by OpKind::ScatterAddRows(idx, adj): d_table[v] = sum of the
// rows of adj whose index is v (kernels/scatter.cu).
//
// Matching: the product's operand dims must pair the one-hot tensor's index
// dims with adj's leading dims in order (batch dims summed by the following
// reduce, the others contracted), the vocabulary dim must be the free dim of
// the one-hot side, and adj must have one more (free) dim.  The one-hot side
// is checked numerically: its cone may only contain element-wise ops, index
// maps, splat constants, iota and one index source; it is evaluated at sampled
// coordinates with synthetic integer indices (including out-of-range ones)
// and must equal [idx == v] everywhere.  A product that fails any check is
// left alone, so the rewrite cannot change what is computed for integral
// index values (Sheaf's token ids).
#include <algorithm>
#include <cmath>
#include <functional>
#include <map>
#include <memory>
#include <random>
#include <set>
#include <string>

#include "ir.h"
#include "plan.h"

namespace sb {
namespace {

struct Matcher {
  const Function& f;
  std::vector<std::vector<int>> users;  // value -> op indices using it

  explicit Matcher(const Function& fn) : f(fn), users(fn.num_values()) {
    for (int i = 0; i < (int)f.ops.size(); ++i)
      for (int o : f.ops[i].operands) users[o].push_back(i);
  }

  const Op* prod(int v) const { return f.producer[v] >= 0 ? &f.ops[f.producer[v]] : nullptr; }

  // Cone of x: every value reachable through allowed ops.  Fails on any other
  // op.  The one non-constant, non-iota leaf is returned in *src.
  bool cone(int x, int* src) const {
    std::set<int> seen;
    std::function<bool(int)> walk = [&](int v) -> bool {
      if (!seen.insert(v).second) return true;
      const Op* p = prod(v);
      if (!p) {  // a parameter: the index source
        if (*src >= 0 && *src != v) return false;
        *src = v;
        return true;
      }
      switch (p->kind) {
        case OpKind::Constant:
          return p->values.size() == 1;
        case OpKind::Iota:
          return true;
        case OpKind::BroadcastInDim: case OpKind::Reshape: case OpKind::Transpose:
          return walk(p->operands[0]);
        default:
          if (!is_elementwise(p->kind)) {
            // any other producer: treated as the index source
            if (*src >= 0 && *src != v) return false;
            *src = v;
            return true;
          }
          for (int o : p->operands)
            if (!walk(o)) return false;
          return true;
      }
    };
    return walk(x) && *src >= 0;
  }

  // Value of x at coordinate c, with the index source replaced by `idx`
  // (row-major over the source's shape).  Double precision; i1 as 0/1.
  double eval(int v, const std::vector<int64_t>& c, int src, const std::vector<double>& idx) const {
    if (v == src) {
      int64_t flat = 0;
      const auto& sh = f.value_types[v].shape;
      for (size_t i = 0; i < sh.size(); ++i) flat = flat * sh[i] + c[i];
      return idx[flat];
    }
    const Op& p = *prod(v);
    const auto& osh = p.type.shape;
    auto arg = [&](int k, const std::vector<int64_t>& cc) { return eval(p.operands[k], cc, src, idx); };
    switch (p.kind) {
      case OpKind::Constant: return p.values[0];
      case OpKind::Iota: return (double)c[p.axis];
      case OpKind::BroadcastInDim: {
        const auto& ish = f.value_types[p.operands[0]].shape;
        std::vector<int64_t> ic(ish.size());
        for (size_t i = 0; i < ish.size(); ++i) ic[i] = ish[i] == 1 ? 0 : c[p.dims[i]];
        return arg(0, ic);
      }
      case OpKind::Transpose: {
        std::vector<int64_t> ic(c.size());
        for (size_t i = 0; i < p.dims.size(); ++i) ic[p.dims[i]] = c[i];
        return arg(0, ic);
      }
      case OpKind::Reshape: {
        const auto& ish = f.value_types[p.operands[0]].shape;
        int64_t lin = 0;
        for (size_t i = 0; i < osh.size(); ++i) lin = lin * osh[i] + c[i];
        std::vector<int64_t> ic(ish.size());
        for (int i = (int)ish.size() - 1; i >= 0; --i) {
          ic[i] = ish[i] ? lin % ish[i] : 0;
          lin = ish[i] ? lin / ish[i] : 0;
        }
        return arg(0, ic);
      }
      default: break;
    }
    std::vector<double> a;
    for (size_t k = 0; k < p.operands.size(); ++k) a.push_back(arg((int)k, c));
    const bool integral = p.type.dtype == DType::I32 || p.type.dtype == DType::I64;
    switch (p.kind) {
      case OpKind::Add: return a[0] + a[1];
      case OpKind::Sub: return a[0] - a[1];
      case OpKind::Mul: return a[0] * a[1];
      case OpKind::Div: return integral ? std::trunc(a[0] / a[1]) : a[0] / a[1];
      case OpKind::Max: return std::max(a[0], a[1]);
      case OpKind::Min: return std::min(a[0], a[1]);
      case OpKind::Abs: return std::fabs(a[0]);
      case OpKind::Neg: return -a[0];
      case OpKind::Sign: return (a[0] > 0) - (a[0] < 0);
      case OpKind::Floor: return std::floor(a[0]);
      case OpKind::Ceil: return std::ceil(a[0]);
      case OpKind::Not: return a[0] == 0 ? 1 : 0;
      case OpKind::And: return (a[0] != 0 && a[1] != 0) ? 1 : 0;
      case OpKind::Or: return (a[0] != 0 || a[1] != 0) ? 1 : 0;
      case OpKind::Convert:
        if (p.type.dtype == DType::I1) return a[0] != 0;
        return integral ? std::trunc(a[0]) : a[0];
      case OpKind::Select: return a[0] != 0 ? a[1] : a[2];
      case OpKind::Clamp: return std::min(std::max(a[1], a[0]), a[2]);
      case OpKind::Compare:
        switch (p.cmp) {
          case CmpDir::EQ: return a[0] == a[1];
          case CmpDir::NE: return a[0] != a[1];
          case CmpDir::LT: return a[0] < a[1];
          case CmpDir::LE: return a[0] <= a[1];
          case CmpDir::GT: return a[0] > a[1];
          case CmpDir::GE: return a[0] >= a[1];
        }
        return NAN;
      default: return NAN;  // not a one-hot cone: the check fails
    }
  }

  // x (shape idx_dims + [V]) equals one_hot(src, V) on sampled coordinates
  // with synthetic integer indices.
  bool is_one_hot(int x, int src) const {
    const auto& xs = f.value_types[x].shape;
    if (xs.size() < 2 || f.value_types[src].numel() * xs.back() != f.value_types[x].numel()) return false;
    std::vector<int64_t> lead(xs.begin(), xs.end() - 1);
    const int64_t V = xs.back(), N = f.value_types[src].numel();
    std::mt19937_64 rng(12345);
    std::vector<double> idx(N);
    for (int64_t i = 0; i < N; ++i) idx[i] = (double)(rng() % (uint64_t)V);
    // a few out-of-range indices: their one-hot rows are zero
    for (int64_t i = 0; i < std::min<int64_t>(N, 4); ++i) idx[(i * 7919) % N] = (i & 1) ? (double)V : -1.0;
    std::vector<int64_t> rows;
    for (int64_t i = 0; i < std::min<int64_t>(N, 24); ++i) rows.push_back(i);
    for (int k = 0; k < 24; ++k) rows.push_back((int64_t)(rng() % (uint64_t)N));
    for (int64_t i = 0; i < std::min<int64_t>(N, 4); ++i) rows.push_back((i * 7919) % N);
    for (int64_t r : rows) {
      std::vector<int64_t> c(xs.size());
      int64_t rem = r;
      for (int d = (int)lead.size() - 1; d >= 0; --d) {
        c[d] = rem % lead[d];
        rem /= lead[d];
      }
      std::vector<int64_t> vs = {0, V - 1};
      const double t = idx[r];
      for (double dv : {t - 1, t, t + 1})
        if (dv >= 0 && dv < V) vs.push_back((int64_t)dv);
      for (int k = 0; k < 6; ++k) vs.push_back((int64_t)(rng() % (uint64_t)V));
      for (int64_t v : vs) {
        c.back() = v;
        const double want = (t == (double)v) ? 1.0 : 0.0;
        if (eval(x, c, src, idx) != want) return false;
      }
    }
    return true;
  }
};

}  // namespace

std::unique_ptr<Function> rewrite_embedding_grad(const Function& f, std::string* log) {
  Matcher m(f);
  std::unique_ptr<Function> g;
  int n_rewritten = 0;
  for (int di = 0; di < (int)f.ops.size(); ++di) {
    const Op& dot = f.ops[di];
    if (dot.kind != OpKind::DotGeneral) continue;
    // left operand: the one-hot tensor x through transposes and reshapes that
    // only insert or drop unit dims; xd[k] = dim of x read by dim k (-1: a
    // unit dim that x does not have)
    int t = dot.operands[0];
    std::vector<int64_t> xd(f.value_types[t].shape.size());
    for (size_t i = 0; i < xd.size(); ++i) xd[i] = (int64_t)i;
    bool chain_ok = true;
    while (m.prod(t) && chain_ok) {
      const Op& p = *m.prod(t);
      if (p.kind == OpKind::Transpose) {
        for (auto& k : xd)
          if (k >= 0) k = p.dims[k];
      } else if (p.kind == OpKind::Reshape) {
        // unit dims only: the non-unit dims keep their order
        const auto& os = p.type.shape;
        const auto& is = f.value_types[p.operands[0]].shape;
        std::vector<int64_t> on, in;
        for (size_t i = 0; i < os.size(); ++i) if (os[i] != 1) on.push_back((int64_t)i);
        for (size_t i = 0; i < is.size(); ++i) if (is[i] != 1) in.push_back((int64_t)i);
        std::vector<int64_t> ext;
        for (auto i : on) ext.push_back(os[i]);
        std::vector<int64_t> ixt;
        for (auto i : in) ixt.push_back(is[i]);
        if (ext != ixt) { chain_ok = false; break; }
        std::vector<int64_t> map(os.size(), -1);
        for (size_t j = 0; j < on.size(); ++j) map[on[j]] = in[j];
        for (auto& k : xd)
          if (k >= 0) k = map[k];
      } else {
        break;
      }
      t = p.operands[0];
    }
    if (!chain_ok) continue;
    const int x = t;
    const auto& xs = f.value_types[x].shape;
    const int r = (int)xs.size() - 1;  // index dims of x; dim r is the vocabulary
    if (r < 1 || f.value_types[x].dtype != DType::F32) continue;
    const int adj = dot.operands[1];
    const auto& as = f.value_types[adj].shape;
    if (f.value_types[adj].dtype != DType::F32) continue;
    const size_t nb = dot.lb.size();
    // the left operand's one free dim is the vocabulary
    {
      int nfree = 0, vfree = -1;
      const auto& ts = f.value_types[dot.operands[0]].shape;
      for (int k = 0; k < (int)ts.size(); ++k)
        if (!std::count(dot.lb.begin(), dot.lb.end(), k) && !std::count(dot.lc.begin(), dot.lc.end(), k) &&
            ts[k] != 1) {
          ++nfree;
          vfree = k;
        }
      if (nfree != 1 || xd[vfree] != r) continue;
    }
    // pairs (x index dim, adj dim) of the batch and contracted dims: every
    // non-unit index dim of x exactly once, in the same order as adj's dims
    std::vector<std::pair<int64_t, int64_t>> pairs;
    bool ok = true;
    for (size_t i = 0; i < nb; ++i) pairs.push_back({xd[dot.lb[i]], dot.rb[i]});
    for (size_t i = 0; i < dot.lc.size(); ++i) pairs.push_back({xd[dot.lc[i]], dot.rc[i]});
    std::vector<int> hit(r, 0);
    for (auto& [a, j] : pairs) {
      if (a < 0) ok = ok && as[j] == 1;  // a unit dim on both sides
      else ok = ok && a < r && !hit[a]++;
    }
    for (int j = 0; j < r && ok; ++j) ok = hit[j] || xs[j] == 1;
    if (!ok) continue;
    {
      std::vector<std::pair<int64_t, int64_t>> sorted;
      for (auto& pr : pairs)
        if (pr.first >= 0) sorted.push_back(pr);
      std::sort(sorted.begin(), sorted.end());
      for (size_t i = 1; i < sorted.size() && ok; ++i) ok = sorted[i].second > sorted[i - 1].second;
    }
    // adj: the paired dims, then its one free dim (D) last
    int adj_free = -1, nfree_adj = 0;
    for (int j = 0; j < (int)as.size(); ++j)
      if (!std::count(dot.rb.begin(), dot.rb.end(), j) && !std::count(dot.rc.begin(), dot.rc.end(), j)) {
        ++nfree_adj;
        adj_free = j;
      }
    if (!ok || nfree_adj != 1 || adj_free != (int)as.size() - 1) continue;
    // batch dims come first in the result and are summed by the reduce
    for (size_t i = 0; i < nb && ok; ++i) ok = dot.lb[i] == (int64_t)i;
    if (!ok) continue;
    // result dims: batch (0..nb-1), vocabulary, adj's free dim
    const int64_t V = xs[r], D = as[adj_free];
    // batched: the only user must be reduce(add, init 0) over dims 0..nb-1
    int replaced = dot.result;
    if (nb > 0) {
      if (m.users[dot.result].size() != 1) continue;
      const Op& red = f.ops[m.users[dot.result][0]];
      if (red.kind != OpKind::Reduce || red.body != ReduceBody::Add || red.operands[0] != dot.result) continue;
      std::vector<int64_t> want;
      for (size_t i = 0; i < nb; ++i) want.push_back((int64_t)i);
      std::vector<int64_t> dims(red.dims.begin(), red.dims.end());
      std::sort(dims.begin(), dims.end());
      const Op* init = m.prod(red.operands[1]);
      if (dims != want || !init || init->kind != OpKind::Constant || init->values.size() != 1 || init->values[0] != 0)
        continue;
      replaced = red.result;
    }
    if (f.value_types[replaced].shape != std::vector<int64_t>{V, D}) continue;
    int src = -1;
    if (!m.cone(x, &src) || !m.is_one_hot(x, src)) continue;
    const DType sdt = f.value_types[src].dtype;
    if (sdt != DType::F32 && sdt != DType::I32) continue;
    if (!g) g = std::make_unique<Function>(f);
    Op s;
    s.kind = OpKind::ScatterAddRows;
    s.result = replaced;
    s.operands = {src, adj};
    s.type = f.value_types[replaced];
    s.line = dot.line;
    g->ops[f.producer[replaced]] = s;
    ++n_rewritten;
  }
  if (g && log) *log = "embedding gradients as row scatter-adds: " + std::to_string(n_rewritten);
  return g;
}

}  // namespace sb
