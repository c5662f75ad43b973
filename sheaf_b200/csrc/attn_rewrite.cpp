// Attention rewrite: finds scaled-dot-product attention in a StableHLO function
// and its reverse-mode gradient, and replaces them by the fused attention ops
// (OpKind::AttnFwd / AttnBwd, kernels/attention.cu).
//
// What Sheaf emits for `causal_self_attention` (sheaf/lib/nn.shf; the softmax
// of sheaf/lib/nn.shf and the tril mask of the builtins, lowered by
// sheaf/src/lowering/stablehlo/emit.rs) is
//     S = dot_general(Q, transpose(K))            [B,H,T,T]
//     M = select(tril != 0, S / c, -1e10)
//     P = exp(M - max(M)) / sum(exp(M - max(M)))  (row-wise over the keys)
//     Y = dot_general(P, V)                       [B,H,T,64]
// and its reverse-mode graph (sheaf/src/autodiff/reverse.rs rules for dot,
// divide, exp, reduce max/sum, select) computes dP = dot(dY, V^T), a chain of
// element-wise and row-reduction ops giving G = dL/dS, then dQ = G K,
// dK = G^T Q, dV = P^T dY.
//
// Matching is structural for the matrix products (operands are followed
// through transposes and tracked by index role: batch b, head h, query q,
// key k, head dim d) and numerical for the element-wise part: the ops between
// S and P (forward) and between (S, dP) and G (backward) must be row-local, and
// are evaluated in double precision on random rows for every query row i; P
// must equal softmax(mask_i(scale * s)) and G must equal
// scale * P * (dP - rowsum(P * dP)).  A region that fails any check is left to
// the generic fusion path, so the rewrite never changes what is computed.
#include <algorithm>
#include <cmath>
#include <map>
#include <random>
#include <set>
#include <stdexcept>

#include "plan.h"

namespace sb {
namespace {

constexpr int HD = 64;

struct Rewriter {
  const Function& f;
  std::vector<char> live;
  std::vector<std::vector<int>> users;  // value -> op indices (live ops)

  explicit Rewriter(const Function& fn) : f(fn) {
    int nv = f.num_values();
    live.assign(nv, 0);
    for (int r : f.returns) live[r] = 1;
    for (int i = (int)f.ops.size() - 1; i >= 0; --i)
      if (live[f.ops[i].result])
        for (int o : f.ops[i].operands) live[o] = 1;
    users.assign(nv, {});
    for (int i = 0; i < (int)f.ops.size(); ++i)
      if (live[f.ops[i].result])
        for (int o : f.ops[i].operands) users[o].push_back(i);
  }

  const Op* prod(int v) const { return f.producer[v] >= 0 ? &f.ops[f.producer[v]] : nullptr; }
  const std::vector<int64_t>& shape(int v) const { return f.value_types[v].shape; }

  // Follows transposes: value dim i == base dim perm[i].
  int resolve(int v, std::vector<int>* perm) const {
    perm->resize(shape(v).size());
    for (size_t i = 0; i < perm->size(); ++i) (*perm)[i] = (int)i;
    for (;;) {
      const Op* op = prod(v);
      if (!op || op->kind != OpKind::Transpose) return v;
      for (auto& p : *perm) p = (int)op->dims[p];
      v = op->operands[0];
    }
  }
};

// ------------------------------------------------------------------ row evaluation
// Evaluates a row-local cone for one (b, h, query i) row in double precision.
// Value classes: [B,H,T,T] -> vector over keys j; [T,T] -> vector (row i);
// [B,H,T] / [B,H,T,1] / scalars -> scalar.
struct Cone {
  const Function& f;
  int64_t B, H, T;
  std::vector<int> leaves;     // values supplied per row (S, dP)
  std::vector<int> order;      // cone values in op order
  std::map<int, int> slot;     // value -> index into the per-row table
  bool ok = true;

  enum Cls { kVec, kScalar, kBad };
  Cls cls(int v) const {
    const auto& s = f.value_types[v].shape;
    if (s == std::vector<int64_t>{B, H, T, T} || s == std::vector<int64_t>{T, T}) return kVec;
    if (s == std::vector<int64_t>{B, H, T} || s == std::vector<int64_t>{B, H, T, 1} || s.empty()) return kScalar;
    return kBad;
  }

  Cone(const Function& fn, int64_t b, int64_t h, int64_t t) : f(fn), B(b), H(h), T(t) {}

  // Collects the cone of `target`, stopping at `leaves`; stop_dot: a
  // dot_general with [B,H,T,T] result that is not a leaf is reported through
  // found_dots instead of failing (used to discover S).
  void build(int target, std::vector<int>* found_dots) {
    std::set<int> seen(leaves.begin(), leaves.end());
    std::vector<int> stack{target}, vals;
    while (!stack.empty()) {
      int v = stack.back();
      stack.pop_back();
      if (seen.count(v)) continue;
      seen.insert(v);
      int pi = f.producer[v];
      if (pi < 0) { ok = false; return; }
      const Op& op = f.ops[pi];
      if (op.kind == OpKind::DotGeneral) {
        if (found_dots && f.value_types[v].shape == std::vector<int64_t>{B, H, T, T}) {
          found_dots->push_back(v);
          continue;
        }
        ok = false;
        return;
      }
      if (cls(v) == kBad) { ok = false; return; }
      vals.push_back(v);
      for (int o : op.operands) stack.push_back(o);
    }
    std::sort(vals.begin(), vals.end(), [&](int a, int b) { return f.producer[a] < f.producer[b]; });
    order = vals;
    int k = 0;
    for (int l : leaves) slot[l] = k++;
    for (int v : order) slot[v] = k++;
  }

  struct RV {
    bool vec = false;
    double s = 0;
    std::vector<double> x;
    double at(int64_t j) const { return vec ? x[j] : s; }
  };

  static double ew1(OpKind k, double a, DType out) {
    switch (k) {
      case OpKind::Tanh: return std::tanh(a);
      case OpKind::Sqrt: return std::sqrt(a);
      case OpKind::Rsqrt: return 1.0 / std::sqrt(a);
      case OpKind::Exp: return std::exp(a);
      case OpKind::Log: return std::log(a);
      case OpKind::Abs: return std::fabs(a);
      case OpKind::Neg: return -a;
      case OpKind::Sin: return std::sin(a);
      case OpKind::Cos: return std::cos(a);
      case OpKind::Not: return a != 0 ? 0.0 : 1.0;
      case OpKind::Sign: return a > 0 ? 1.0 : (a < 0 ? -1.0 : a);
      case OpKind::Floor: return std::floor(a);
      case OpKind::Ceil: return std::ceil(a);
      case OpKind::Logistic: return 1.0 / (1.0 + std::exp(-a));
      case OpKind::Convert:
        if (out == DType::I1) return a != 0 ? 1.0 : 0.0;
        if (!dtype_is_float(out)) return std::trunc(a);
        return a;
      default: return NAN;
    }
  }
  static double ew2(const Op& op, double a, double b) {
    switch (op.kind) {
      case OpKind::Add: return a + b;
      case OpKind::Sub: return a - b;
      case OpKind::Mul: return a * b;
      case OpKind::Div: return a / b;
      case OpKind::Pow: return std::pow(a, b);
      case OpKind::Max: return std::max(a, b);
      case OpKind::Min: return std::min(a, b);
      case OpKind::Rem: return std::fmod(a, b);
      case OpKind::And: return (a != 0 && b != 0) ? 1.0 : 0.0;
      case OpKind::Or: return (a != 0 || b != 0) ? 1.0 : 0.0;
      case OpKind::Compare:
        switch (op.cmp) {
          case CmpDir::EQ: return a == b;
          case CmpDir::NE: return a != b;
          case CmpDir::LT: return a < b;
          case CmpDir::LE: return a <= b;
          case CmpDir::GT: return a > b;
          case CmpDir::GE: return a >= b;
        }
        return NAN;
      default: return NAN;
    }
  }

  // Evaluates row i; leaf rows in `leaf_rows` (same order as leaves).
  // Returns false when an op is not row-local.
  bool eval(int64_t i, const std::vector<std::vector<double>>& leaf_rows, std::vector<RV>* tab) const {
    tab->assign(slot.size(), RV{});
    for (size_t l = 0; l < leaves.size(); ++l) {
      (*tab)[l].vec = true;
      (*tab)[l].x = leaf_rows[l];
    }
    auto get = [&](int v) -> const RV* {
      auto it = slot.find(v);
      return it == slot.end() ? nullptr : &(*tab)[it->second];
    };
    for (int v : order) {
      const Op& op = f.ops[f.producer[v]];
      RV& r = (*tab)[slot.at(v)];
      const auto& rs = op.type.shape;
      const bool vec_out = cls(v) == kVec;
      std::vector<const RV*> in;
      for (int o : op.operands) {
        const RV* p = get(o);
        if (!p) return false;
        in.push_back(p);
      }
      auto same_shape_dims = [&](const std::vector<int64_t>& want) { return op.dims == want; };
      switch (op.kind) {
        case OpKind::Constant:
          if (op.values.size() != 1) return false;
          r.s = op.values[0];
          break;
        case OpKind::Iota: {
          int64_t ax = op.axis;
          bool tt = rs.size() == 2;
          int64_t qd = tt ? 0 : 2, kd = tt ? 1 : 3;
          if (rs.size() == 3 && ax == 2) { r.s = (double)i; break; }
          if (!vec_out) return false;
          if (ax == qd) { r.s = (double)i; break; }
          if (ax != kd) return false;
          r.vec = true;
          r.x.resize(T);
          for (int64_t j = 0; j < T; ++j) r.x[j] = (double)j;
          break;
        }
        case OpKind::BroadcastInDim: {
          const auto& is = f.value_types[op.operands[0]].shape;
          bool okb = false;
          if (is.empty()) okb = true;
          else if (is == rs) okb = true;  // identity or same-shape permutation-free broadcast
          else if (is == std::vector<int64_t>{T, T} && rs.size() == 4) okb = same_shape_dims({2, 3});
          else if (is == std::vector<int64_t>{B, H, T, 1} && rs.size() == 4) okb = same_shape_dims({0, 1, 2, 3});
          else if (is == std::vector<int64_t>{B, H, T} && rs.size() == 4) okb = same_shape_dims({0, 1, 2});
          else if (is == std::vector<int64_t>{B, H, T} && rs.size() == 4 && rs[3] == 1) okb = same_shape_dims({0, 1, 2});
          if (is == rs) {
            for (size_t d = 0; d < op.dims.size(); ++d) okb = okb && op.dims[d] == (int64_t)d;
          }
          if (!okb) return false;
          r = *in[0];
          break;
        }
        case OpKind::Reshape: {
          const auto& is = f.value_types[op.operands[0]].shape;
          if (!(is == rs || (cls(op.operands[0]) == kScalar && cls(v) == kScalar && !is.empty() && !rs.empty())))
            return false;
          r = *in[0];
          break;
        }
        case OpKind::Reduce: {
          if (!(cls(v) == kScalar && !rs.empty() && op.dims == std::vector<int64_t>{3} &&
                f.value_types[op.operands[0]].shape == std::vector<int64_t>{B, H, T, T}))
            return false;
          double acc = in[1]->s;
          for (int64_t j = 0; j < T; ++j) {
            double x = in[0]->at(j);
            switch (op.body) {
              case ReduceBody::Add: acc += x; break;
              case ReduceBody::Max: acc = std::max(acc, x); break;
              case ReduceBody::Min: acc = std::min(acc, x); break;
              case ReduceBody::Mul: acc *= x; break;
            }
          }
          r.s = acc;
          break;
        }
        case OpKind::Select: case OpKind::Clamp: {
          bool any_vec = in[0]->vec || in[1]->vec || in[2]->vec;
          auto f3 = [&](double a, double b, double c) {
            return op.kind == OpKind::Select ? (a != 0 ? b : c) : std::min(std::max(b, a), c);
          };
          if (!any_vec) { r.s = f3(in[0]->s, in[1]->s, in[2]->s); break; }
          r.vec = true;
          r.x.resize(T);
          for (int64_t j = 0; j < T; ++j) r.x[j] = f3(in[0]->at(j), in[1]->at(j), in[2]->at(j));
          break;
        }
        default: {
          if (is_unary_elementwise(op.kind)) {
            if (!in[0]->vec) { r.s = ew1(op.kind, in[0]->s, op.type.dtype); break; }
            r.vec = true;
            r.x.resize(T);
            for (int64_t j = 0; j < T; ++j) r.x[j] = ew1(op.kind, in[0]->x[j], op.type.dtype);
            break;
          }
          if (is_binary_elementwise(op.kind) || op.kind == OpKind::Compare) {
            if (!in[0]->vec && !in[1]->vec) { r.s = ew2(op, in[0]->s, in[1]->s); break; }
            r.vec = true;
            r.x.resize(T);
            for (int64_t j = 0; j < T; ++j) r.x[j] = ew2(op, in[0]->at(j), in[1]->at(j));
            break;
          }
          return false;
        }
      }
      if (vec_out && !r.vec) {  // a broadcast scalar stays a scalar; fine for vector classes
      }
    }
    return true;
  }

  // Scalar value of a constant-only cone member (e.g. sqrt(64)).
  bool scalar_of(int v, double* out) const {
    Cone c(f, B, H, T);
    c.build(v, nullptr);
    if (!c.ok) return false;
    std::vector<RV> tab;
    if (!c.eval(0, {}, &tab)) return false;
    const RV& r = tab[c.slot.at(v)];
    if (r.vec) return false;
    *out = r.s;
    return true;
  }
};

// Reference rows used by the numerical checks.
void softmax_row(const std::vector<double>& s, double scale, bool causal, int64_t i, std::vector<double>* p) {
  int64_t T = (int64_t)s.size();
  p->assign(T, 0.0);
  double m = -INFINITY;
  for (int64_t j = 0; j < T; ++j)
    if (!causal || j <= i) m = std::max(m, scale * s[j]);
  double sum = 0;
  for (int64_t j = 0; j < T; ++j)
    if (!causal || j <= i) sum += ((*p)[j] = std::exp(scale * s[j] - m));
  for (auto& x : *p) x /= sum;
}

bool close_rows(const Cone::RV& got, const std::vector<double>& want, double tol) {
  double mag = 0;
  for (double w : want) mag = std::max(mag, std::fabs(w));
  for (size_t j = 0; j < want.size(); ++j) {
    double g = got.at((int64_t)j);
    if (!(std::fabs(g - want[j]) <= tol * (1.0 + mag))) return false;
  }
  return true;
}

// Rows checked: every row (the mask is a function of the row index).
std::vector<int64_t> check_rows(int64_t T) {
  std::vector<int64_t> r(T);
  for (int64_t i = 0; i < T; ++i) r[i] = i;
  return r;
}

struct Labels {
  int base = -1;
  std::vector<char> lab;  // per base dim
};

struct FwdMatch {
  int y_op = -1;           // op index of dot(P, V)
  int y = -1, P = -1, S = -1;
  int64_t B = 0, H = 0, T = 0;
  double scale = 1;
  bool causal = false;
  Labels q, k, v;          // bases of Q, K, V with index roles
  std::vector<int> cone;   // values between S and P (inclusive of P)
};

struct BwdMatch {
  int dq = -1, dk = -1, dv = -1;      // values of the three gradient dot_generals
  std::vector<char> dq_lab, dk_lab, dv_lab;  // index roles of their result dims
  int dP = -1;
  Labels dy;
};

// Labels of a dot operand's dims, given the labels of its base.
bool operand_labels(const Rewriter& rw, int v, const Labels& L, std::vector<char>* out) {
  std::vector<int> perm;
  int base = rw.resolve(v, &perm);
  if (base != L.base) return false;
  out->resize(perm.size());
  for (size_t i = 0; i < perm.size(); ++i) (*out)[i] = L.lab[perm[i]];
  return true;
}

// Index roles of a dot_general's result, or empty when the batch/contracting
// roles do not pair up.
std::vector<char> dot_result_labels(const Op& op, const std::vector<char>& la, const std::vector<char>& lb) {
  std::vector<char> res;
  for (size_t i = 0; i < op.lb.size(); ++i) {
    if (la[op.lb[i]] != lb[op.rb[i]]) return {};
    res.push_back(la[op.lb[i]]);
  }
  for (size_t i = 0; i < op.lc.size(); ++i)
    if (la[op.lc[i]] != lb[op.rc[i]]) return {};
  for (size_t d = 0; d < la.size(); ++d)
    if (!std::count(op.lb.begin(), op.lb.end(), (int64_t)d) && !std::count(op.lc.begin(), op.lc.end(), (int64_t)d))
      res.push_back(la[d]);
  for (size_t d = 0; d < lb.size(); ++d)
    if (!std::count(op.rb.begin(), op.rb.end(), (int64_t)d) && !std::count(op.rc.begin(), op.rc.end(), (int64_t)d))
      res.push_back(lb[d]);
  return res;
}

bool is_perm_of(const std::vector<char>& a, const std::string& want) {
  std::string s(a.begin(), a.end()), w = want;
  std::sort(s.begin(), s.end());
  std::sort(w.begin(), w.end());
  return s == w;
}

Labels labels_of(const Rewriter& rw, int v, const std::vector<char>& dim_roles) {
  std::vector<int> perm;
  Labels L;
  L.base = rw.resolve(v, &perm);
  L.lab.assign(perm.size(), '?');
  for (size_t i = 0; i < perm.size(); ++i) L.lab[perm[i]] = dim_roles[i];
  return L;
}

bool match_forward(const Rewriter& rw, int op_index, FwdMatch* m) {
  const Function& f = rw.f;
  const Op& y = f.ops[op_index];
  if (y.kind != OpKind::DotGeneral || !rw.live[y.result]) return false;
  const auto& ys = y.type.shape;
  if (ys.size() != 4 || ys[3] != HD || y.type.dtype != DType::F32) return false;
  if (y.lb != std::vector<int64_t>{0, 1} || y.rb != std::vector<int64_t>{0, 1} || y.lc != std::vector<int64_t>{3} ||
      y.rc != std::vector<int64_t>{2})
    return false;
  int64_t B = ys[0], H = ys[1], T = ys[2];
  if (T < 128 || T % 128) return false;
  int P = y.operands[0], V = y.operands[1];
  if (rw.shape(P) != std::vector<int64_t>{B, H, T, T} || rw.shape(V) != std::vector<int64_t>{B, H, T, HD}) return false;
  // cone P <- S
  Cone probe(f, B, H, T);
  std::vector<int> dots;
  probe.build(P, &dots);
  if (!probe.ok || dots.size() != 1) return false;
  int S = dots[0];
  const Op& so = f.ops[f.producer[S]];
  if (so.lb != std::vector<int64_t>{0, 1} || so.rb != std::vector<int64_t>{0, 1} || so.lc != std::vector<int64_t>{3})
    return false;
  if (rw.shape(so.operands[0]) != std::vector<int64_t>{B, H, T, HD}) return false;
  std::vector<char> kroles;
  if (so.rc == std::vector<int64_t>{2} && rw.shape(so.operands[1]) == std::vector<int64_t>{B, H, HD, T})
    kroles = {'b', 'h', 'd', 'k'};
  else if (so.rc == std::vector<int64_t>{3} && rw.shape(so.operands[1]) == std::vector<int64_t>{B, H, T, HD})
    kroles = {'b', 'h', 'k', 'd'};
  else
    return false;
  Cone cone(f, B, H, T);
  cone.leaves = {S};
  cone.build(P, nullptr);
  if (!cone.ok) return false;
  // scale: the op of the cone that consumes S
  double scale = 1;
  int n_use = 0;
  for (int v : cone.order) {
    const Op& op = f.ops[f.producer[v]];
    for (size_t s = 0; s < op.operands.size(); ++s) {
      if (op.operands[s] != S) continue;
      ++n_use;
      if (op.kind == OpKind::Div && s == 0) {
        double c;
        if (!cone.scalar_of(op.operands[1], &c) || c == 0) return false;
        scale = 1.0 / c;
      } else if (op.kind == OpKind::Mul) {
        double c;
        if (!cone.scalar_of(op.operands[1 - s], &c)) return false;
        scale = c;
      }
    }
  }
  if (n_use != 1) return false;
  // numerical check, causal first
  std::mt19937_64 rng(0x5eedULL);
  std::normal_distribution<double> nd(0.0, 2.0);
  bool found = false, causal = false;
  for (int hyp = 0; hyp < 2 && !found; ++hyp) {
    causal = hyp == 0;
    bool good = true;
    std::vector<Cone::RV> tab;
    std::vector<double> srow(T), want;
    for (int64_t i : check_rows(T)) {
      for (auto& x : srow) x = nd(rng);
      if (!cone.eval(i, {srow}, &tab)) return false;
      softmax_row(srow, scale, causal, i, &want);
      if (!close_rows(tab[cone.slot.at(P)], want, 1e-9)) { good = false; break; }
    }
    found = good;
  }
  if (!found) return false;
  m->y_op = op_index;
  m->y = y.result;
  m->P = P;
  m->S = S;
  m->B = B;
  m->H = H;
  m->T = T;
  m->scale = scale;
  m->causal = causal;
  m->q = labels_of(rw, so.operands[0], {'b', 'h', 'q', 'd'});
  m->k = labels_of(rw, so.operands[1], kroles);
  m->v = labels_of(rw, V, {'b', 'h', 'k', 'd'});
  m->cone = cone.order;
  return true;
}

bool match_backward(const Rewriter& rw, const FwdMatch& m, BwdMatch* bm) {
  const Function& f = rw.f;
  const std::vector<int64_t> bhtt{m.B, m.H, m.T, m.T};
  Labels Pl{m.P, {'b', 'h', 'q', 'k'}};
  // dP = dot(dY, V^T): result roles (b, h, q, k)
  int dP = -1;
  Labels dy;
  for (const Op& op : f.ops) {
    if (op.kind != OpKind::DotGeneral || !rw.live[op.result] || op.result == m.S || op.type.shape != bhtt) continue;
    std::vector<char> lv;
    if (!operand_labels(rw, op.operands[1], m.v, &lv)) continue;
    if (op.lb.size() != 2 || op.lc.size() != 1) continue;
    // dY roles: batch dims take V's batch roles, the contracted dim is d, the free dim q
    const auto& xs = rw.shape(op.operands[0]);
    if (xs.size() != 4) continue;
    std::vector<char> lx(4, 'q');
    for (size_t i = 0; i < op.lb.size(); ++i) lx[op.lb[i]] = lv[op.rb[i]];
    lx[op.lc[0]] = lv[op.rc[0]];
    if (lv[op.rc[0]] != 'd') continue;
    std::vector<char> res = dot_result_labels(op, lx, lv);
    if (res != std::vector<char>{'b', 'h', 'q', 'k'}) continue;
    if (dP >= 0) return false;  // ambiguous
    dP = op.result;
    dy = labels_of(rw, op.operands[0], lx);
  }
  if (dP < 0) return false;
  // dV = P^T dY, dQ = G K, dK = G^T Q
  int dv = -1, dq = -1, dk = -1, G = -1;
  std::vector<char> dv_lab, dq_lab, dk_lab;
  for (const Op& op : f.ops) {
    if (op.kind != OpKind::DotGeneral || !rw.live[op.result] || op.type.shape.size() != 4) continue;
    if (op.result == m.y) continue;
    for (int sw = 0; sw < 2; ++sw) {
      int a = op.operands[sw], b = op.operands[1 - sw];
      std::vector<char> la, lb;
      auto res_of = [&](const std::vector<char>& x, const std::vector<char>& y) {
        return sw == 0 ? dot_result_labels(op, x, y) : dot_result_labels(op, y, x);
      };
      // dV
      if (operand_labels(rw, a, Pl, &la) && operand_labels(rw, b, dy, &lb)) {
        auto r = res_of(la, lb);
        if (!r.empty() && is_perm_of(r, "bhkd") && r[0] == 'b' && r[1] == 'h') {
          if (dv >= 0) return false;
          dv = op.result;
          dv_lab = r;
        }
      }
      // dQ / dK: the other operand is a [B,H,T,T] value G (roles b,h,q,k)
      std::vector<int> gp;
      int gb = rw.resolve(a, &gp);
      if (gb == m.P || gb == m.S || gb == dP || rw.shape(gb) != bhtt) continue;
      Labels Gl{gb, {'b', 'h', 'q', 'k'}};
      if (!operand_labels(rw, a, Gl, &la)) continue;
      if (operand_labels(rw, b, m.k, &lb)) {
        auto r = res_of(la, lb);
        if (!r.empty() && is_perm_of(r, "bhqd") && r[0] == 'b' && r[1] == 'h') {
          if (dq >= 0 || (G >= 0 && G != gb)) return false;
          dq = op.result;
          dq_lab = r;
          G = gb;
        }
      }
      if (operand_labels(rw, b, m.q, &lb)) {
        auto r = res_of(la, lb);
        if (!r.empty() && is_perm_of(r, "bhkd") && r[0] == 'b' && r[1] == 'h') {
          if (dk >= 0 || (G >= 0 && G != gb)) return false;
          dk = op.result;
          dk_lab = r;
          G = gb;
        }
      }
    }
  }
  if (dv < 0 || dq < 0 || dk < 0 || G < 0) return false;
  // G must be dL/dS: scale * P * (dP - rowsum(P * dP)), row-locally from (S, dP)
  Cone cone(f, m.B, m.H, m.T);
  cone.leaves = {m.S, dP};
  cone.build(G, nullptr);
  if (!cone.ok) return false;
  std::mt19937_64 rng(0xa77eULL);
  std::normal_distribution<double> nd(0.0, 2.0), nd1(0.0, 1.0);
  std::vector<Cone::RV> tab;
  std::vector<double> srow(m.T), drow(m.T), p, want(m.T);
  for (int64_t i : check_rows(m.T)) {
    for (auto& x : srow) x = nd(rng);
    for (auto& x : drow) x = nd1(rng);
    if (!cone.eval(i, {srow, drow}, &tab)) return false;
    softmax_row(srow, m.scale, m.causal, i, &p);
    double D = 0;
    for (int64_t j = 0; j < m.T; ++j) D += p[j] * drow[j];
    for (int64_t j = 0; j < m.T; ++j) want[j] = m.scale * p[j] * (drow[j] - D);
    if (!close_rows(tab[cone.slot.at(G)], want, 1e-9)) return false;
  }
  // the inputs of the fused backward must exist before the first gradient dot
  int ip = std::min({f.producer[dq], f.producer[dk], f.producer[dv]});
  for (int base : {dy.base, m.q.base, m.k.base, m.v.base})
    if (f.producer[base] >= ip) return false;
  if (m.y_op >= ip) return false;
  bm->dq = dq;
  bm->dk = dk;
  bm->dv = dv;
  bm->dq_lab = dq_lab;
  bm->dk_lab = dk_lab;
  bm->dv_lab = dv_lab;
  bm->dP = dP;
  bm->dy = dy;
  return true;
}

// Builds the rewritten function.
struct Builder {
  Function g;
  std::vector<std::vector<Op>> before;  // ops inserted before original op i
  std::map<int, std::vector<Op>> replace;  // original op index -> ops producing its result

  explicit Builder(const Function& f) : g(f) { before.assign(f.ops.size() + 1, {}); }

  int new_value(const Type& t) {
    g.value_types.push_back(t);
    return (int)g.value_types.size() - 1;
  }
  static Op mk(OpKind k, int result, std::vector<int> operands, Type t) {
    Op op;
    op.kind = k;
    op.result = result;
    op.operands = std::move(operands);
    op.type = std::move(t);
    return op;
  }
  Type f32(std::vector<int64_t> s) {
    Type t;
    t.shape = std::move(s);
    t.dtype = DType::F32;
    return t;
  }
  // transpose of `base` into the dim order `want` (roles), given base roles
  int canonical(std::vector<Op>* ops, const Labels& L, const std::string& want) {
    std::vector<int64_t> perm;
    for (char c : want) {
      auto it = std::find(L.lab.begin(), L.lab.end(), c);
      if (it == L.lab.end()) throw std::runtime_error("internal: attention role missing");
      perm.push_back(it - L.lab.begin());
    }
    bool ident = true;
    for (size_t i = 0; i < perm.size(); ++i) ident = ident && perm[i] == (int64_t)i;
    if (ident) return L.base;
    std::vector<int64_t> s;
    for (auto p : perm) s.push_back(g.value_types[L.base].shape[p]);
    int v = new_value(f32(s));
    Op op = mk(OpKind::Transpose, v, {L.base}, f32(s));
    op.dims = perm;
    ops->push_back(op);
    return v;
  }
  // slice [lo, hi) of a 1-D packed buffer, reshaped to `shape`
  int part(std::vector<Op>* ops, int packed, int64_t lo, int64_t hi, std::vector<int64_t> shape, int result = -1) {
    int s = new_value(f32({hi - lo}));
    Op sl = mk(OpKind::Slice, s, {packed}, f32({hi - lo}));
    sl.a0 = {lo};
    sl.a1 = {hi};
    sl.a2 = {1};
    ops->push_back(sl);
    int r = result >= 0 ? result : new_value(f32(shape));
    ops->push_back(mk(OpKind::Reshape, r, {s}, f32(shape)));
    return r;
  }
  // value `result` with roles `roles` from a [B,T,H,64] buffer `src` (roles b x h d, x = q or k)
  void from_bthd(std::vector<Op>* ops, int src, char x, const std::vector<char>& roles, int result) {
    const char have[4] = {'b', x, 'h', 'd'};
    std::vector<int64_t> perm, shape;
    for (char c : roles) {
      int d = (int)(std::find(have, have + 4, c) - have);
      perm.push_back(d);
      shape.push_back(g.value_types[src].shape[d]);
    }
    Op op = mk(OpKind::Transpose, result, {src}, f32(shape));
    op.dims = perm;
    ops->push_back(op);
  }

  Function finish(const Function& f) {
    std::vector<Op> out;
    for (size_t i = 0; i < f.ops.size(); ++i) {
      for (auto& op : before[i]) out.push_back(op);
      auto it = replace.find((int)i);
      if (it == replace.end()) out.push_back(f.ops[i]);
      else for (auto& op : it->second) out.push_back(op);
    }
    g.ops = std::move(out);
    g.producer.assign(g.value_types.size(), -1);
    for (size_t i = 0; i < g.ops.size(); ++i) g.producer[g.ops[i].result] = (int)i;
    return std::move(g);
  }
};

}  // namespace

std::unique_ptr<Function> rewrite_attention(const Function& f, std::string* log) {
  Rewriter rw(f);
  std::vector<FwdMatch> fwd;
  for (int i = 0; i < (int)f.ops.size(); ++i) {
    FwdMatch m;
    if (f.ops[i].kind == OpKind::DotGeneral && match_forward(rw, i, &m)) fwd.push_back(m);
  }
  if (fwd.empty()) return nullptr;
  Builder bld(f);
  int n_fwd = 0, n_bwd = 0;
  for (const FwdMatch& m : fwd) {
    BwdMatch bm;
    bool bwd = match_backward(rw, m, &bm);
    if (!bwd) {
      // forward only: the region's values must have no other use
      std::set<int> region(m.cone.begin(), m.cone.end());
      region.insert(m.S);
      bool other = false;
      for (int v : region) {
        for (int ui : rw.users[v]) {
          int r = f.ops[ui].result;
          if (!region.count(r) && ui != m.y_op) other = true;
        }
        if (std::count(f.returns.begin(), f.returns.end(), v)) other = true;
      }
      if (other) continue;
    }
    const int64_t B = m.B, H = m.H, T = m.T, N = B * T * H * HD, R = B * H * T;
    // forward, at the position of dot(P, V)
    std::vector<Op> fw;
    int qc = bld.canonical(&fw, m.q, "bhqd"), kc = bld.canonical(&fw, m.k, "bhkd"),
        vc = bld.canonical(&fw, m.v, "bhkd");
    int pf = bld.new_value(bld.f32({N + R}));
    Op af = Builder::mk(OpKind::AttnFwd, pf, {qc, kc, vc}, bld.f32({N + R}));
    af.values = {m.scale};
    af.axis = m.causal ? 1 : 0;
    fw.push_back(af);
    int yb = bld.part(&fw, pf, 0, N, {B, T, H, HD});
    bld.from_bthd(&fw, yb, 'q', {'b', 'h', 'q', 'd'}, m.y);
    int lse = bld.part(&fw, pf, N, N + R, {B, H, T});
    bld.replace[m.y_op] = fw;
    ++n_fwd;
    if (!bwd) continue;
    // backward, before the first of the three gradient products
    int ip = std::min({f.producer[bm.dq], f.producer[bm.dk], f.producer[bm.dv]});
    std::vector<Op>& pre = bld.before[ip];
    int q2 = bld.canonical(&pre, m.q, "bhqd"), k2 = bld.canonical(&pre, m.k, "bhkd"),
        v2 = bld.canonical(&pre, m.v, "bhkd"), dyc = bld.canonical(&pre, bm.dy, "bhqd");
    // dQ, dK, dV interleaved per token: (B,T,3,H,64), so the three gradients
    // are adjacent column blocks of one [B*T, 3*H*64] matrix (the layout of
    // the fused projection whose slices produced q, k, v)
    int pb = bld.new_value(bld.f32({3 * N + R}));
    Op ab = Builder::mk(OpKind::AttnBwd, pb, {q2, k2, v2, dyc, m.y, lse}, bld.f32({3 * N + R}));
    ab.values = {m.scale};
    ab.axis = af.axis;
    pre.push_back(ab);
    int g5 = bld.part(&pre, pb, 0, 3 * N, {B, T, 3, H, HD});
    auto channel = [&](int c) {
      int s = bld.new_value(bld.f32({B, T, 1, H, HD}));
      Op sl = Builder::mk(OpKind::Slice, s, {g5}, bld.f32({B, T, 1, H, HD}));
      sl.a0 = {0, 0, c, 0, 0};
      sl.a1 = {B, T, c + 1, H, HD};
      sl.a2 = {1, 1, 1, 1, 1};
      pre.push_back(sl);
      int r = bld.new_value(bld.f32({B, T, H, HD}));
      pre.push_back(Builder::mk(OpKind::Reshape, r, {s}, bld.f32({B, T, H, HD})));
      return r;
    };
    int dqb = channel(0), dkb = channel(1), dvb = channel(2);
    std::vector<Op> rq, rk, rv;
    bld.from_bthd(&rq, dqb, 'q', bm.dq_lab, bm.dq);
    bld.from_bthd(&rk, dkb, 'k', bm.dk_lab, bm.dk);
    bld.from_bthd(&rv, dvb, 'k', bm.dv_lab, bm.dv);
    bld.replace[f.producer[bm.dq]] = rq;
    bld.replace[f.producer[bm.dk]] = rk;
    bld.replace[f.producer[bm.dv]] = rv;
    ++n_bwd;
  }
  if (!n_fwd) return nullptr;
  if (log) *log = "attention: " + std::to_string(n_fwd) + " forward, " + std::to_string(n_bwd) + " backward";
  return std::make_unique<Function>(bld.finish(f));
}

}  // namespace sb
