// Sibling-GEMM merging: a graph rewrite that runs before planning.
//
// Sheaf's GPT attention block (examples/nanoGPT/model.shf, causal-self-
// attention) slices the fused c_attn weight into W_q, W_k, W_v and multiplies
// the same activation by each, so reverse mode yields three forward GEMMs of
// width D, three input-gradient GEMMs that are summed, three weight-gradient
// GEMMs and a sum of zero-pads that reassembles dW (the adjoint of the
// slices).  Once the fused attention backward writes dQ, dK, dV interleaved
// per token, every one of these groups reads adjacent blocks of one buffer:
//   A  dots sharing one operand whose other operands are adjacent blocks along
//      a free dim  ->  one dot over the union, the siblings slice its result
//      (also through a reduce_add over batch dims: the weight gradients);
//   B  a sum of dots whose operands are adjacent blocks along one contracting
//      dim  ->  one dot over the union of the contraction;
//   C  a sum of zero-pads of slices that tile a value  ->  that value.
// The union of adjacent blocks is expressed as an OpKind::StridedView of the
// blocks' common base buffer.
#include <algorithm>
#include <map>
#include <set>
#include <tuple>

#include "plan.h"

namespace sb {
namespace {

struct IrView {
  int base = -1;
  int64_t off = 0;
  std::vector<int64_t> shape, str;
  bool same_layout(const IrView& o) const { return base == o.base && shape == o.shape && str == o.str; }
  bool operator==(const IrView& o) const { return same_layout(o) && off == o.off; }
};

void normalize(IrView* v) {
  for (size_t i = 0; i < v->shape.size(); ++i)
    if (v->shape[i] == 1) v->str[i] = 0;
}

bool contiguous(const IrView& v) {
  const auto rm = row_major(v.shape);
  for (size_t i = 0; i < v.shape.size(); ++i)
    if (v.shape[i] != 1 && v.str[i] != rm[i]) return false;
  return true;
}

bool is_zero_splat(const Function& g, int v) {
  const int p = g.producer[v];
  return p >= 0 && g.ops[p].kind == OpKind::Constant && g.ops[p].values.size() == 1 && g.ops[p].values[0] == 0.0;
}

std::vector<int64_t> free_dims(int64_t rank, const std::vector<int64_t>& batch, const std::vector<int64_t>& contr) {
  std::vector<int64_t> r;
  for (int64_t d = 0; d < rank; ++d)
    if (!std::count(batch.begin(), batch.end(), d) && !std::count(contr.begin(), contr.end(), d)) r.push_back(d);
  return r;
}

class Merger {
 public:
  explicit Merger(const Function& f) : g_(f) {}

  // Applies one merge; false when none applies.
  bool step() {
    index();
    return merge_shared_operand() || merge_contraction_sum() || merge_pad_sum();
  }
  Function take() {
    dce();
    return std::move(g_);
  }
  int merged_a = 0, merged_b = 0, merged_c = 0;

 private:
  Function g_;
  std::vector<int> uses_;
  std::vector<char> returned_;
  std::vector<std::vector<int>> users_;  // value -> consuming op indices
  std::map<int, IrView> memo_;

  const Type& type(int v) const { return g_.value_types[v]; }
  const Op* producer(int v) const { return g_.producer[v] >= 0 ? &g_.ops[g_.producer[v]] : nullptr; }

  void index() {
    g_.producer.assign(g_.num_values(), -1);
    for (size_t i = 0; i < g_.ops.size(); ++i) g_.producer[g_.ops[i].result] = (int)i;
    uses_.assign(g_.num_values(), 0);
    users_.assign(g_.num_values(), {});
    returned_.assign(g_.num_values(), 0);
    for (int r : g_.returns) returned_[r] = 1;
    for (size_t i = 0; i < g_.ops.size(); ++i)
      for (int o : g_.ops[i].operands) {
        ++uses_[o];
        users_[o].push_back((int)i);
      }
    memo_.clear();
  }
  bool single(int v) const { return uses_[v] == 1 && !returned_[v]; }

  // View of v over the row-major layout of the nearest value that is not a
  // slice, transpose, no-copy reshape or strided view.
  IrView view(int v) {
    auto it = memo_.find(v);
    if (it != memo_.end()) return it->second;
    IrView r;
    bool done = false;
    if (const Op* op = producer(v)) {
      switch (op->kind) {
        case OpKind::Slice: {
          r = view(op->operands[0]);
          for (size_t i = 0; i < r.shape.size(); ++i) {
            r.off += op->a0[i] * r.str[i];
            r.str[i] *= op->a2[i];
          }
          r.shape = op->type.shape;
          done = true;
          break;
        }
        case OpKind::Transpose: {
          const IrView in = view(op->operands[0]);
          r = in;
          r.shape = op->type.shape;
          for (size_t i = 0; i < op->dims.size(); ++i) r.str[i] = in.str[op->dims[i]];
          done = true;
          break;
        }
        case OpKind::Reshape: {
          const IrView in = view(op->operands[0]);
          std::vector<int64_t> ns;
          if (reshape_view(in.shape, in.str, op->type.shape, &ns)) {
            r = in;
            r.shape = op->type.shape;
            r.str = ns;
            done = true;
          }
          break;
        }
        case OpKind::StridedView: {
          const IrView in = view(op->operands[0]);
          if (contiguous(in)) {
            r.base = in.base;
            r.off = in.off + op->a0[0];
            r.shape = op->type.shape;
            r.str = op->a2;
            done = true;
          }
          break;
        }
        default:
          break;
      }
    }
    if (!done) {
      r.base = v;
      r.off = 0;
      r.shape = type(v).shape;
      r.str = row_major(r.shape);
    }
    normalize(&r);
    memo_[v] = r;
    return r;
  }

  int new_value(const Type& t) {
    g_.value_types.push_back(t);
    return g_.num_values() - 1;
  }
  Op strided(int result, const IrView& v, DType dt) {
    Op op;
    op.kind = OpKind::StridedView;
    op.result = result;
    op.operands = {v.base};
    op.type.shape = v.shape;
    op.type.dtype = dt;
    op.a0 = {v.off};
    op.a2 = v.str;
    return op;
  }
  Op zero_const(int result, DType dt) {
    Op op;
    op.kind = OpKind::Constant;
    op.result = result;
    op.type.dtype = dt;
    op.values = {0.0};
    return op;
  }
  Op slice_of(int src, int result, const Type& t, int64_t dim, int64_t lo, int64_t hi) {
    Op op;
    op.kind = OpKind::Slice;
    op.result = result;
    op.operands = {src};
    op.type = t;
    const auto& ss = type(src).shape;
    op.a0.assign(ss.size(), 0);
    op.a1 = ss;
    op.a2.assign(ss.size(), 1);
    op.a0[dim] = lo;
    op.a1[dim] = hi;
    return op;
  }

  // Rebuilds the op list: `insert` goes before op index `at`, ops in
  // `replace` are swapped for their new form, ops in `erase` are dropped.
  void rebuild(int at, const std::vector<Op>& insert, const std::map<int, Op>& replace, const std::set<int>& erase) {
    std::vector<Op> out;
    out.reserve(g_.ops.size() + insert.size());
    for (int i = 0; i < (int)g_.ops.size(); ++i) {
      if (i == at)
        for (const Op& op : insert) out.push_back(op);
      if (erase.count(i)) continue;
      auto it = replace.find(i);
      out.push_back(it != replace.end() ? it->second : g_.ops[i]);
    }
    g_.ops = std::move(out);
    g_.producer.assign(g_.num_values(), -1);
    for (size_t i = 0; i < g_.ops.size(); ++i) g_.producer[g_.ops[i].result] = (int)i;
  }

  // ---- A: shared operand, the other operand split along a free dim
  struct Unit {
    int dot = -1, red = -1;  // op indices (red: reduce_add over the dot, or -1)
  };
  bool unit_of(int di, Unit* u) {
    const Op& d = g_.ops[di];
    u->dot = di;
    u->red = -1;
    if (!single(d.result)) return true;
    const int ci = users_[d.result][0];
    const Op& c = g_.ops[ci];
    if (c.kind == OpKind::Reduce && c.body == ReduceBody::Add && c.operands.size() == 2 && c.operands[0] == d.result &&
        is_zero_splat(g_, c.operands[1]))
      u->red = ci;
    return true;
  }

  bool merge_shared_operand() {
    using Key = std::tuple<int, std::vector<int64_t>, std::vector<int64_t>, std::vector<int64_t>,
                           std::vector<int64_t>, std::vector<int64_t>, int, std::vector<int64_t>,
                           std::vector<int64_t>, int64_t, std::vector<int64_t>, std::vector<int64_t>, int>;
    std::map<Key, std::vector<std::pair<int64_t, Unit>>> groups;
    for (int i = 0; i < (int)g_.ops.size(); ++i) {
      const Op& d = g_.ops[i];
      if (d.kind != OpKind::DotGeneral || d.type.dtype != DType::F32) continue;
      Unit u;
      unit_of(i, &u);
      const std::vector<int64_t> rdims = u.red >= 0 ? g_.ops[u.red].dims : std::vector<int64_t>{-1};
      for (int s = 0; s < 2; ++s) {
        const IrView sh = view(d.operands[s]), ot = view(d.operands[1 - s]);
        Key k{s, d.lb, d.rb, d.lc, d.rc, rdims, sh.base, sh.shape, sh.str, sh.off, ot.shape, ot.str, ot.base};
        groups[k].push_back({ot.off, u});
      }
    }
    for (auto& [k, members] : groups) {
      if (members.size() < 2) continue;
      std::sort(members.begin(), members.end(), [](const auto& a, const auto& b) { return a.first < b.first; });
      const int s = std::get<0>(k);
      const Op& d0 = g_.ops[members[0].second.dot];
      const int other = 1 - s;
      const IrView ov = view(d0.operands[other]);
      const auto fd = free_dims((int64_t)ov.shape.size(), other == 0 ? d0.lb : d0.rb, other == 0 ? d0.lc : d0.rc);
      for (int64_t f : fd) {
        const int64_t step = ov.shape[f] * ov.str[f];
        if (ov.str[f] <= 0 || step <= 0) continue;
        // longest run of consecutive blocks starting anywhere
        size_t b = 0;
        while (b < members.size()) {
          size_t e = b + 1;
          while (e < members.size() && members[e].first == members[e - 1].first + step &&
                 (members[e].second.red >= 0) == (members[b].second.red >= 0))
            ++e;
          if (e - b >= 2 && apply_shared(std::vector<std::pair<int64_t, Unit>>(members.begin() + b,
                                                                                 members.begin() + e),
                                         s, f))
            return true;
          b = e;
        }
      }
    }
    return false;
  }

  bool apply_shared(const std::vector<std::pair<int64_t, Unit>>& run, int s, int64_t f) {
    const int n = (int)run.size();
    const int other = 1 - s;
    // the first unit in program order supplies the shared operand
    int first = 0;
    for (int j = 1; j < n; ++j)
      if (run[j].second.dot < run[first].second.dot) first = j;
    const Op d0 = g_.ops[run[first].second.dot];
    const bool red = run[0].second.red >= 0;
    // output position of free dim f of the split operand
    const int64_t nb = (int64_t)d0.lb.size();
    const auto lf = free_dims((int64_t)type(d0.operands[0]).shape.size(), d0.lb, d0.lc);
    const auto rf = free_dims((int64_t)type(d0.operands[1]).shape.size(), d0.rb, d0.rc);
    const auto& mine = other == 0 ? lf : rf;
    const int64_t pos_out = nb + (other == 0 ? 0 : (int64_t)lf.size()) +
                            (int64_t)(std::find(mine.begin(), mine.end(), f) - mine.begin());
    int64_t pos_fin = pos_out;
    if (red) {
      const auto& rd = g_.ops[run[0].second.red].dims;
      if (std::count(rd.begin(), rd.end(), pos_out)) return false;
      for (auto x : rd)
        if (x < pos_out) --pos_fin;
    }
    IrView all = view(d0.operands[other]);
    all.off = run[0].first;
    all.shape[f] *= n;
    std::vector<Op> ins;
    Type vt;
    vt.shape = all.shape;
    vt.dtype = type(d0.operands[other]).dtype;
    const int ov = new_value(vt);
    ins.push_back(strided(ov, all, vt.dtype));
    Op dot = d0;
    dot.operands[other] = ov;
    dot.type.shape[pos_out] *= n;
    dot.result = new_value(dot.type);
    ins.push_back(dot);
    int fin = dot.result;
    if (red) {
      Op r = g_.ops[run[first].second.red];
      const int z = new_value(Type{{}, r.type.dtype});
      ins.push_back(zero_const(z, r.type.dtype));
      r.operands = {dot.result, z};
      r.type.shape[pos_fin] *= n;
      r.result = new_value(r.type);
      ins.push_back(r);
      fin = r.result;
    }
    int at = (int)g_.ops.size();
    for (const auto& m : run) at = std::min(at, m.second.dot);
    std::map<int, Op> replace;
    std::set<int> erase;
    const int64_t e = type(fin).shape[pos_fin] / n;
    for (int j = 0; j < n; ++j) {
      const Unit& u = run[j].second;
      const int last = red ? u.red : u.dot;
      const Op& lo = g_.ops[last];
      replace[last] = slice_of(fin, lo.result, lo.type, pos_fin, j * e, (j + 1) * e);
      if (red) erase.insert(u.dot);
    }
    rebuild(at, ins, replace, erase);
    ++merged_a;
    return true;
  }

  // ---- B: sum of dots over adjacent blocks of one contracting dim
  void add_leaves(int v, std::vector<int>* leaves, std::vector<int>* adds) {
    const Op* p = producer(v);
    if (p && p->kind == OpKind::Add && single(v)) {
      adds->push_back(g_.producer[v]);
      for (int o : p->operands) add_leaves(o, leaves, adds);
    } else {
      leaves->push_back(v);
    }
  }
  bool is_tree_root(int i) const {
    const Op& a = g_.ops[i];
    if (a.kind != OpKind::Add) return false;
    if (!single(a.result)) return true;
    return g_.ops[users_[a.result][0]].kind != OpKind::Add;
  }

  bool merge_contraction_sum() {
    for (int i = 0; i < (int)g_.ops.size(); ++i) {
      if (!is_tree_root(i)) continue;
      const Op& root = g_.ops[i];
      std::vector<int> leaves, adds{i};
      for (int o : root.operands) add_leaves(o, &leaves, &adds);
      if (leaves.size() < 2) continue;
      const Op* d0 = producer(leaves[0]);
      bool ok = d0 && d0->kind == OpKind::DotGeneral;
      for (int l : leaves) {
        const Op* d = producer(l);
        ok = ok && d && d->kind == OpKind::DotGeneral && single(l) && d->lb == d0->lb && d->rb == d0->rb &&
             d->lc == d0->lc && d->rc == d0->rc && d->type == d0->type && d->type == root.type;
      }
      if (!ok) continue;
      struct Leaf { IrView l, r; int op; };
      std::vector<Leaf> lv;
      for (int l : leaves) {
        const Op* d = producer(l);
        lv.push_back({view(d->operands[0]), view(d->operands[1]), g_.producer[l]});
      }
      for (const Leaf& x : lv) ok = ok && x.l.same_layout(lv[0].l) && x.r.same_layout(lv[0].r);
      if (!ok) continue;
      std::sort(lv.begin(), lv.end(), [](const Leaf& a, const Leaf& b) { return a.l.off < b.l.off; });
      const int n = (int)lv.size();
      for (size_t j = 0; j < d0->lc.size(); ++j) {
        const int64_t cl = d0->lc[j], cr = d0->rc[j];
        const int64_t sl = lv[0].l.shape[cl] * lv[0].l.str[cl], sr = lv[0].r.shape[cr] * lv[0].r.str[cr];
        if (lv[0].l.str[cl] <= 0 || lv[0].r.str[cr] <= 0) continue;
        bool run = true;
        for (int k = 1; k < n; ++k)
          run = run && lv[k].l.off == lv[k - 1].l.off + sl && lv[k].r.off == lv[k - 1].r.off + sr;
        if (!run) continue;
        IrView la = lv[0].l, ra = lv[0].r;
        la.shape[cl] *= n;
        ra.shape[cr] *= n;
        const Op& dd = g_.ops[lv[0].op];
        std::vector<Op> ins;
        Type lt{la.shape, type(dd.operands[0]).dtype}, rt{ra.shape, type(dd.operands[1]).dtype};
        const int lvv = new_value(lt), rvv = new_value(rt);
        ins.push_back(strided(lvv, la, lt.dtype));
        ins.push_back(strided(rvv, ra, rt.dtype));
        Op dot = dd;
        dot.operands = {lvv, rvv};
        dot.result = root.result;
        std::map<int, Op> replace{{i, dot}};
        std::set<int> erase(adds.begin() + 1, adds.end());
        for (const Leaf& x : lv) erase.insert(x.op);
        rebuild(i, ins, replace, erase);
        ++merged_b;
        return true;
      }
    }
    return false;
  }

  // ---- C: sum of zero-pads of slices that tile one value
  bool merge_pad_sum() {
    for (int i = 0; i < (int)g_.ops.size(); ++i) {
      if (!is_tree_root(i)) continue;
      const Op& root = g_.ops[i];
      std::vector<int> leaves, adds{i};
      for (int o : root.operands) add_leaves(o, &leaves, &adds);
      if (leaves.size() < 2) continue;
      int M = -1;
      int64_t dim = -1;
      std::vector<std::pair<int64_t, int64_t>> ranges;
      bool ok = true;
      for (int l : leaves) {
        const Op* p = producer(l);
        if (!p || p->kind != OpKind::Pad || !single(l) || !is_zero_splat(g_, p->operands[1])) { ok = false; break; }
        const Op* sl = producer(p->operands[0]);
        if (!sl || sl->kind != OpKind::Slice) { ok = false; break; }
        const int m = sl->operands[0];
        if (M >= 0 && m != M) { ok = false; break; }
        M = m;
        if (!(type(M) == root.type)) { ok = false; break; }
        const auto& ms = type(M).shape;
        int64_t d = -1;
        for (size_t k = 0; k < ms.size() && ok; ++k) {
          ok = ok && sl->a2[k] == 1 && p->a2[k] == 0;
          if (sl->a0[k] != 0 || sl->a1[k] != ms[k]) {
            if (d >= 0) ok = false;
            d = (int64_t)k;
          }
          ok = ok && p->a0[k] == sl->a0[k] && p->a1[k] == ms[k] - sl->a1[k];
        }
        if (!ok || d < 0 || (dim >= 0 && d != dim)) { ok = false; break; }
        dim = d;
        ranges.push_back({sl->a0[d], sl->a1[d]});
      }
      if (!ok) continue;
      std::sort(ranges.begin(), ranges.end());
      int64_t at = 0;
      for (auto& r : ranges) {
        ok = ok && r.first == at;
        at = r.second;
      }
      if (!ok || at != type(M).shape[dim]) continue;
      // uses of the sum now read M
      const int old = root.result;
      for (Op& op : g_.ops)
        for (int& o : op.operands)
          if (o == old) o = M;
      for (int& r : g_.returns)
        if (r == old) r = M;
      std::set<int> erase(adds.begin(), adds.end());
      rebuild(-1, {}, {}, erase);
      ++merged_c;
      return true;
    }
    return false;
  }

  void dce() {
    for (int iter = 0; iter < 64; ++iter) {
      index();
      std::set<int> dead;
      for (int i = 0; i < (int)g_.ops.size(); ++i)
        if (uses_[g_.ops[i].result] == 0 && !returned_[g_.ops[i].result]) dead.insert(i);
      if (dead.empty()) break;
      rebuild(-1, {}, {}, dead);
    }
  }
};

}  // namespace

std::unique_ptr<Function> merge_sibling_dots(const Function& f, std::string* log) {
  Merger m(f);
  int n = 0;
  while (n < 4096 && m.step()) ++n;
  if (!n) return nullptr;
  if (log)
    *log = "merged GEMMs: " + std::to_string(m.merged_a) + " shared-operand, " + std::to_string(m.merged_b) +
           " contraction, " + std::to_string(m.merged_c) + " pad-sum";
  return std::make_unique<Function>(m.take());
}

}  // namespace sb
