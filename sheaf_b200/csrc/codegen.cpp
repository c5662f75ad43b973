// Kernel text generation for fused clusters.  Each cluster node is evaluated at
// a coordinate tuple (C integer expressions); index maps (broadcast, transpose,
// reshape, slice, reverse, pad, concatenate, gather) rewrite the tuple, and
// elementwise nodes combine operand values.  Values are memoized per
// (node, coordinates) so a node shared inside one cluster is computed once.
#include "codegen.h"

#include <functional>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <stdexcept>

namespace sb {

const char* ctype_of(DType t) {
  switch (t) {
    case DType::F32: return "float";
    case DType::BF16: return "float";
    case DType::F64: return "double";
    case DType::I32: return "int";
    case DType::I64: return "long long";
    case DType::I1: return "bool";
  }
  return "float";
}

// Element type in memory: bf16 values are stored as their 16 bits and
// computed on as f32.
const char* mtype_of(DType t) { return t == DType::BF16 ? "unsigned short" : ctype_of(t); }

// x rounded to bf16 (round to nearest even on the f32 value; NaN and
// infinities pass through).
double bf16_round(double x) {
  float f = (float)x;
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) return x;
  u = (u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u;
  std::memcpy(&f, &u, 4);
  return f;
}

namespace {

constexpr int kDup = -2, kConst = -3, kParam = -4;
constexpr int kThreads = 256;
constexpr int64_t kMaxGrid = 148 * 16;

std::string join(const std::vector<std::string>& v, const char* sep) {
  std::string s;
  for (size_t i = 0; i < v.size(); ++i) {
    if (i) s += sep;
    s += v[i];
  }
  return s;
}

std::string f32_literal(double x) {
  float f = (float)x;
  uint32_t u;
  std::memcpy(&u, &f, 4);
  char buf[48];
  std::snprintf(buf, sizeof buf, "__int_as_float(0x%08x)", u);
  return buf;
}

std::string literal(double x, const std::string& ctype) {
  if (ctype == "float") return f32_literal(x);
  if (ctype == "bool") return x != 0 ? "true" : "false";
  // i32 constants wrap modulo 2^32 (a seed's 32-bit halves arrive as 0..2^32-1)
  if (ctype == "int") return "(int)" + std::to_string((uint32_t)(uint64_t)(int64_t)x) + "u";
  if (ctype == "double") {
    char buf[48];
    std::snprintf(buf, sizeof buf, "%.17g", x);
    return buf;
  }
  return std::to_string((long long)x) + (ctype == "long long" ? "LL" : "");
}

// coordinate arithmetic helpers that keep literal zeros simple
std::string c_mul(const std::string& c, int64_t k) {
  if (c == "0" || k == 0) return "0";
  if (k == 1) return c;
  return "(" + c + ")*" + std::to_string(k);
}
std::string c_add(const std::string& a, const std::string& b) {
  if (a == "0") return b;
  if (b == "0") return a;
  return a + "+" + b;
}

// Raised while generating a 4-wide loop when some access uses the lane
// coordinate other than as the innermost index of a contiguous f32 read; the
// loop is then generated one element per thread.
struct VecFail {};

const char* const kLane[4] = {"cL", "(cL+1)", "(cL+2)", "(cL+3)"};

// Programmatic dependent launch: every generated kernel is launched so that it
// may start while the previous kernel in the stream finishes; it first waits
// for that kernel's results, then lets the next kernel start launching.
const char* const kPdlPrologue =
    "  asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");\n"
    "  asm volatile(\"griddepcontrol.launch_dependents;\");\n";

// Lane coordinates of 4-wide code: "<b>" or "(<b>+k)", k = 1..3, where the
// base b is "cL" (one float4 group per thread) or "cL<j>" (chunk j of a row
// held in registers by a row group).  Returns k and the base, or -1.
int lane_of(const std::string& s, std::string* base = nullptr) {
  auto is_base = [](const std::string& b) {
    if (b.size() < 2 || b[0] != 'c' || b[1] != 'L') return false;
    for (size_t i = 2; i < b.size(); ++i)
      if (b[i] < '0' || b[i] > '9') return false;
    return true;
  };
  if (is_base(s)) {
    if (base) *base = s;
    return 0;
  }
  if (s.size() > 5 && s.front() == '(' && s.back() == ')') {
    const size_t plus = s.find('+');
    if (plus == std::string::npos || plus + 3 != s.size()) return -1;
    const std::string b = s.substr(1, plus - 1);
    const char k = s[plus + 1];
    if (!is_base(b) || k < '1' || k > '3') return -1;
    if (base) *base = b;
    return k - '0';
  }
  return -1;
}

std::string lane_coord(const std::string& base, int k) {
  return k == 0 ? base : "(" + base + "+" + std::to_string(k) + ")";
}

bool uses_lane(const std::string& s) { return s.find("cL") != std::string::npos; }

}  // namespace

bool CodeGen::is_materialized_for(const Ctx& c, int v) const {
  int cl = cluster_[v];
  if (cl == kParam || cl == kConst) return true;
  return cl == v && v != c.root;
}

std::string CodeGen::index_type(const Op& root, int64_t extra) const {
  int64_t mx = std::max(root.type.numel(), extra);
  for (auto& t : f_.value_types) mx = std::max(mx, t.numel());
  return mx >= (int64_t(1) << 31) - 1 ? "long long" : "int";
}

CodeGen::Val CodeGen::leaf_load(Ctx& c, int v, const std::vector<std::string>& coords) {
  auto rit = c.reg_kind.find(v);
  if (rit != c.reg_kind.end()) {
    // an earlier row-group member's output: its registers
    std::string key = std::to_string(v) + "@row";
    if (rit->second == 0) {
      std::string base;
      const int k = coords.empty() ? -1 : lane_of(coords.back(), &base);
      if (k < 0) throw VecFail{};
      key = std::to_string(v) + "@" + base + ":" + std::to_string(k);
    }
    auto it2 = c.regs.find(key);
    if (it2 == c.regs.end()) throw VecFail{};
    return it2->second;
  }
  auto it = c.leaf_index.find(v);
  int li;
  if (it == c.leaf_index.end()) {
    li = (int)c.leaves.size();
    c.leaves.push_back(v);
    c.leaf_index[v] = li;
  } else {
    li = it->second;
  }
  const Type& t = f_.value_types[v];
  auto st = row_major(t.shape);
  if (c.vec) {
    int lane = -1;
    std::string base = "cL";
    for (size_t i = 0; i < coords.size(); ++i) {
      if (!uses_lane(coords[i])) continue;
      if (i + 1 != coords.size() || (lane = lane_of(coords[i], &base)) < 0) throw VecFail{};
    }
    if (lane >= 0) {
      // innermost index is the lane coordinate itself: lanes 0..3 read 4
      // consecutive floats starting at a multiple of 4 (row-major leaf whose
      // innermost extent is a multiple of 4, lane 0 coordinate cL % 4 == 0)
      if ((t.dtype != DType::F32 && t.dtype != DType::BF16) || t.shape.back() % 4 || c.memo.size() > 1)
        throw VecFail{};
      std::string off0 = "0";
      for (size_t i = 0; i + 1 < coords.size(); ++i) off0 = c_add(off0, c_mul(coords[i], st[i]));
      off0 = c_add(off0, base);
      const std::string key = std::to_string(li) + ":" + off0;
      auto vit = c.vloads.find(key);
      std::string var;
      if (vit == c.vloads.end()) {
        var = fresh(c, "v");
        if (t.dtype == DType::BF16)  // 4 bf16 in 8 bytes, widened
          c.body << c.pad() << "const float4 " << var << " = sb_bf16x4(*(const uint2*)(L" << li << " + " << off0
                 << "));\n";
        else
          c.body << c.pad() << "const float4 " << var << " = *(const float4*)(L" << li << " + " << off0 << ");\n";
        c.vloads[key] = var;
      } else {
        var = vit->second;
      }
      return Val{var + "." + "xyzw"[lane], "float"};
    }
  }
  std::string off = "0";
  for (size_t i = 0; i < coords.size(); ++i) off = c_add(off, c_mul(coords[i], st[i]));
  Val r{fresh(c), ctype_of(t.dtype)};
  if (t.dtype == DType::BF16)
    c.body << c.pad() << "const float " << r.name << " = sb_bf16_ld(L" << li << "[" << off << "]);\n";
  else
    c.body << c.pad() << "const " << r.ctype << " " << r.name << " = L" << li << "[" << off << "];\n";
  return r;
}

CodeGen::Val CodeGen::eval(Ctx& c, int v, const std::vector<std::string>& coords) {
  std::string key = std::to_string(v) + "@" + join(coords, ",");
  for (int s = (int)c.memo.size() - 1; s >= 0; --s) {
    auto it = c.memo[s].find(key);
    if (it != c.memo[s].end()) return it->second;
  }
  Val out;
  if (is_materialized_for(c, v)) {
    out = leaf_load(c, v, coords);
    c.memo.back()[key] = out;
    return out;
  }
  int pi = f_.producer[v];
  if (pi < 0) throw std::runtime_error("codegen: value without producer is not materialized");
  const Op& op = f_.ops[pi];
  if (!(cluster_[v] == c.root || cluster_[v] == kDup))
    throw std::runtime_error(std::string("codegen: node outside cluster (") + opkind_name(op.kind) + ")");
  std::string ct = ctype_of(op.type.dtype);
  // bf16 arithmetic: each op's f32 result is rounded to bf16 (round to
  // nearest even), as an op on bf16 tensors produces bf16 values
  const bool bf = op.type.dtype == DType::BF16;
  auto emit = [&](const std::string& expr) {
    Val r{fresh(c), ct};
    c.body << c.pad() << "const " << ct << " " << r.name << " = " << (bf ? "sb_bf16_rn(" + expr + ")" : expr)
           << ";\n";
    return r;
  };
  // integer a OP b modulo 2^width, computed unsigned (no signed overflow)
  auto wrap = [&](const std::string& a, const char* o, const std::string& b) {
    if (ct == "int") return "(int)((unsigned)(" + a + ") " + o + " (unsigned)(" + b + "))";
    if (ct == "long long")
      return "(long long)((unsigned long long)(" + a + ") " + o + " (unsigned long long)(" + b + "))";
    return a + " " + o + " " + b;
  };
  const auto& osh = op.type.shape;
  switch (op.kind) {
    case OpKind::Constant:
      out = Val{literal(bf ? bf16_round(op.values[0]) : op.values[0], ct), ct};
      break;
    case OpKind::Iota:
      out = emit("(" + ct + ")(" + coords[op.axis] + ")");
      break;
    case OpKind::BroadcastInDim: {
      const auto& ish = f_.value_types[op.operands[0]].shape;
      std::vector<std::string> ic(ish.size());
      for (size_t i = 0; i < ish.size(); ++i)
        ic[i] = (ish[i] == 1 && osh[op.dims[i]] != 1) ? "0" : coords[op.dims[i]];
      out = eval(c, op.operands[0], ic);
      break;
    }
    case OpKind::Transpose: {
      std::vector<std::string> ic(op.dims.size());
      for (size_t i = 0; i < op.dims.size(); ++i) ic[op.dims[i]] = coords[i];
      out = eval(c, op.operands[0], ic);
      break;
    }
    case OpKind::Reshape: {
      const auto& ish = f_.value_types[op.operands[0]].shape;
      std::vector<int64_t> inz, outz;
      std::vector<size_t> outpos;
      for (auto d : ish) if (d != 1) inz.push_back(d);
      for (size_t i = 0; i < osh.size(); ++i) if (osh[i] != 1) { outz.push_back(osh[i]); outpos.push_back(i); }
      std::vector<std::string> ic(ish.size(), "0");
      if (inz == outz) {
        size_t k = 0;
        for (size_t i = 0; i < ish.size(); ++i) if (ish[i] != 1) ic[i] = coords[outpos[k++]];
      } else {
        if (c.vec)
          for (auto& x : coords)
            if (uses_lane(x)) throw VecFail{};
        auto so = row_major(osh);
        std::string lin = "0";
        for (size_t i = 0; i < osh.size(); ++i) lin = c_add(lin, c_mul(coords[i], so[i]));
        std::string ln = fresh(c, "lin");
        c.body << c.pad() << "const " << c.idx << " " << ln << " = " << lin << ";\n";
        auto si = row_major(ish);
        for (size_t i = 0; i < ish.size(); ++i) {
          if (ish[i] == 1) continue;
          std::string e = si[i] == 1 ? ln : "(" + ln + "/" + std::to_string(si[i]) + ")";
          bool first_nontrivial = true;
          for (size_t j = 0; j < i; ++j) if (ish[j] != 1) first_nontrivial = false;
          if (!first_nontrivial) e = "(" + e + "%" + std::to_string(ish[i]) + ")";
          ic[i] = e;
        }
      }
      out = eval(c, op.operands[0], ic);
      break;
    }
    case OpKind::Slice: {
      std::vector<std::string> ic(coords.size());
      for (size_t i = 0; i < coords.size(); ++i)
        ic[i] = c_add(std::to_string(op.a0[i]) == "0" ? "0" : std::to_string(op.a0[i]), c_mul(coords[i], op.a2[i]));
      out = eval(c, op.operands[0], ic);
      break;
    }
    case OpKind::StridedView: {
      // flat position in the operand's row-major layout, split into its coords
      if (c.vec)
        for (auto& x : coords)
          if (uses_lane(x)) throw VecFail{};
      const auto& ish = f_.value_types[op.operands[0]].shape;
      std::string lin = std::to_string(op.a0[0]);
      for (size_t i = 0; i < osh.size(); ++i) lin = c_add(lin, c_mul(coords[i], op.a2[i]));
      std::string ln = fresh(c, "lin");
      c.body << c.pad() << "const " << c.idx << " " << ln << " = " << lin << ";\n";
      const auto si = row_major(ish);
      std::vector<std::string> ic(ish.size(), "0");
      bool first = true;
      for (size_t i = 0; i < ish.size(); ++i) {
        if (ish[i] == 1) continue;
        std::string e = si[i] == 1 ? ln : "(" + ln + "/" + std::to_string(si[i]) + ")";
        if (!first) e = "(" + e + "%" + std::to_string(ish[i]) + ")";
        first = false;
        ic[i] = e;
      }
      out = eval(c, op.operands[0], ic);
      break;
    }
    case OpKind::Reverse: {
      std::vector<std::string> ic = coords;
      for (auto d : op.dims) ic[d] = "(" + std::to_string(osh[d] - 1) + "-(" + coords[d] + "))";
      out = eval(c, op.operands[0], ic);
      break;
    }
    case OpKind::Pad: {
      const auto& ish = f_.value_types[op.operands[0]].shape;
      Val pv = eval(c, op.operands[1], {});
      out = Val{fresh(c), ct};
      c.body << c.pad() << ct << " " << out.name << " = " << pv.name << ";\n";
      std::vector<std::string> conds, ic(ish.size());
      for (size_t i = 0; i < ish.size(); ++i) {
        int64_t step = op.a2[i] + 1;
        std::string rel = "(" + coords[i] + "-(" + std::to_string(op.a0[i]) + "))";
        conds.push_back(rel + ">=0");
        conds.push_back(rel + "<" + std::to_string((ish[i] - 1) * step + 1));
        if (step != 1) {
          conds.push_back(rel + "%" + std::to_string(step) + "==0");
          ic[i] = "(" + rel + "/" + std::to_string(step) + ")";
        } else {
          ic[i] = rel;
        }
      }
      c.body << c.pad() << "if (" << (conds.empty() ? "true" : join(conds, " && ")) << ") {\n";
      c.indent++;
      c.memo.emplace_back();
      Val in = eval(c, op.operands[0], ic);
      c.body << c.pad() << out.name << " = " << in.name << ";\n";
      c.memo.pop_back();
      c.indent--;
      c.body << c.pad() << "}\n";
      break;
    }
    case OpKind::Concatenate: {
      out = Val{fresh(c), ct};
      c.body << c.pad() << ct << " " << out.name << ";\n";
      int64_t base = 0;
      for (size_t j = 0; j < op.operands.size(); ++j) {
        int64_t ext = f_.value_types[op.operands[j]].shape[op.axis];
        std::vector<std::string> ic = coords;
        ic[op.axis] = "(" + coords[op.axis] + "-" + std::to_string(base) + ")";
        bool last = j + 1 == op.operands.size();
        c.body << c.pad() << (j ? "else " : "") << (last ? "{\n" : "if ((" + coords[op.axis] + ")<" + std::to_string(base + ext) + ") {\n");
        c.indent++;
        c.memo.emplace_back();
        Val in = eval(c, op.operands[j], ic);
        c.body << c.pad() << out.name << " = " << in.name << ";\n";
        c.memo.pop_back();
        c.indent--;
        c.body << c.pad() << "}\n";
        base += ext;
      }
      break;
    }
    case OpKind::Gather: {
      if (c.vec)
        for (auto& x : coords)
          if (uses_lane(x)) throw VecFail{};
      const auto& tsh = f_.value_types[op.operands[0]].shape;
      const auto& ish = f_.value_types[op.operands[1]].shape;
      int ivd = (int)op.axis;
      std::vector<std::string> batch;
      for (size_t d = 0; d < osh.size(); ++d)
        if (!std::count(op.offset_dims.begin(), op.offset_dims.end(), (int64_t)d)) batch.push_back(coords[d]);
      std::vector<std::string> starts(tsh.size(), "0");
      int64_t nidx = ivd < (int)ish.size() ? ish[ivd] : 1;
      for (int64_t k = 0; k < (int64_t)op.start_index_map.size() && k < nidx; ++k) {
        std::vector<std::string> icoord;
        size_t b = 0;
        for (size_t d = 0; d < ish.size(); ++d) icoord.push_back((int)d == ivd ? std::to_string(k) : batch[b++]);
        if (ivd >= (int)ish.size()) { /* implicit trailing index dim */ }
        Val iv = eval(c, op.operands[1], icoord);
        int64_t od = op.start_index_map[k];
        int64_t hi = tsh[od] - op.slice_sizes[od];
        std::string s = fresh(c, "g");
        c.body << c.pad() << "const " << c.idx << " " << s << " = min(max((" << c.idx << ")(" << iv.name
               << "), (" << c.idx << ")0), (" << c.idx << ")" << hi << ");\n";
        starts[od] = s;
      }
      std::vector<std::string> tc(tsh.size());
      size_t oo = 0;
      std::vector<std::string> offs;
      for (auto d : op.offset_dims) offs.push_back(coords[d]);
      for (size_t d = 0; d < tsh.size(); ++d) {
        if (std::count(op.collapsed.begin(), op.collapsed.end(), (int64_t)d)) tc[d] = starts[d];
        else tc[d] = c_add(starts[d], offs[oo++]);
      }
      out = eval(c, op.operands[0], tc);
      break;
    }
    case OpKind::Select: {
      Val p = eval(c, op.operands[0], coords);
      Val a = eval(c, op.operands[1], coords);
      Val b = eval(c, op.operands[2], coords);
      out = emit("(" + p.name + " ? " + a.name + " : " + b.name + ")");
      break;
    }
    case OpKind::Clamp: {
      Val lo = eval(c, op.operands[0], f_.value_types[op.operands[0]].shape.empty() ? std::vector<std::string>{} : coords);
      Val x = eval(c, op.operands[1], coords);
      Val hi = eval(c, op.operands[2], f_.value_types[op.operands[2]].shape.empty() ? std::vector<std::string>{} : coords);
      if (ct == "float") out = emit("fminf(fmaxf(" + x.name + ", " + lo.name + "), " + hi.name + ")");
      else out = emit("min(max(" + x.name + ", " + lo.name + "), " + hi.name + ")");
      break;
    }
    case OpKind::Compare: {
      Val a = eval(c, op.operands[0], coords);
      Val b = eval(c, op.operands[1], coords);
      static const char* ops[] = {"==", "!=", "<", "<=", ">", ">="};
      out = emit("(" + a.name + " " + ops[(int)op.cmp] + " " + b.name + ")");
      break;
    }
    case OpKind::Bitcast: {
      Val a = eval(c, op.operands[0], coords);
      if (a.ctype == ct) out = a;
      else if (ct == "int") out = emit("__float_as_int(" + a.name + ")");
      else out = emit("__int_as_float(" + a.name + ")");
      break;
    }
    case OpKind::Convert: {
      Val a = eval(c, op.operands[0], coords);
      if (ct == "bool") out = emit("(" + a.name + " != 0)");
      else if (a.ctype == "bool") out = emit("(" + a.name + " ? (" + ct + ")1 : (" + ct + ")0)");
      else out = emit("(" + ct + ")(" + a.name + ")");
      break;
    }
    default: {
      if (is_binary_elementwise(op.kind)) {
        Val a = eval(c, op.operands[0], coords);
        Val b = eval(c, op.operands[1], coords);
        const std::string& x = a.name;
        const std::string& y = b.name;
        bool fl = ct == "float" || ct == "double";
        switch (op.kind) {
          // integers wrap modulo 2^width (two's complement), as StableHLO defines
          case OpKind::Add: out = emit(fl ? x + " + " + y : wrap(x, "+", y)); break;
          case OpKind::Sub: out = emit(fl ? x + " - " + y : wrap(x, "-", y)); break;
          case OpKind::Mul: out = emit(fl ? x + " * " + y : wrap(x, "*", y)); break;
          case OpKind::Div: out = emit(fl ? x + " / " + y : "(" + y + " != 0 ? " + x + " / " + y + " : 0)"); break;
          case OpKind::Pow: out = emit(fl ? "powf(" + x + ", " + y + ")" : "(" + ct + ")powf((float)" + x + ", (float)" + y + ")"); break;
          case OpKind::Max: out = emit(fl ? "fmaxf(" + x + ", " + y + ")" : "max(" + x + ", " + y + ")"); break;
          case OpKind::Min: out = emit(fl ? "fminf(" + x + ", " + y + ")" : "min(" + x + ", " + y + ")"); break;
          case OpKind::Rem: out = emit(fl ? "fmodf(" + x + ", " + y + ")" : "(" + y + " != 0 ? " + x + " % " + y + " : 0)"); break;
          case OpKind::And: out = emit(ct == "bool" ? x + " && " + y : x + " & " + y); break;
          case OpKind::Or: out = emit(ct == "bool" ? x + " || " + y : x + " | " + y); break;
          default: throw std::runtime_error("codegen: unhandled binary op");
        }
      } else if (is_unary_elementwise(op.kind)) {
        Val a = eval(c, op.operands[0], coords);
        const std::string& x = a.name;
        switch (op.kind) {
          case OpKind::Tanh: out = emit("tanhf(" + x + ")"); break;
          case OpKind::Sqrt: out = emit("sqrtf(" + x + ")"); break;
          case OpKind::Rsqrt: out = emit("rsqrtf(" + x + ")"); break;
          case OpKind::Exp: out = emit("expf(" + x + ")"); break;
          case OpKind::Log: out = emit("logf(" + x + ")"); break;
          case OpKind::Abs:
            out = emit(ct == "float" ? "fabsf(" + x + ")" : "(" + x + " < 0 ? " + wrap("0", "-", x) + " : " + x + ")");
            break;
          case OpKind::Neg: out = emit(ct == "float" || ct == "double" ? "-" + x : wrap("0", "-", x)); break;
          case OpKind::Sin: out = emit("sinf(" + x + ")"); break;
          case OpKind::Cos: out = emit("cosf(" + x + ")"); break;
          case OpKind::Not: out = emit(ct == "bool" ? "!" + x : "~" + x); break;
          case OpKind::Sign:
            out = emit(ct == "float" ? "(" + x + " > 0.f ? 1.f : (" + x + " < 0.f ? -1.f : " + x + "))"
                                     : "((" + x + " > 0) - (" + x + " < 0))");
            break;
          case OpKind::Floor: out = emit("floorf(" + x + ")"); break;
          case OpKind::Ceil: out = emit("ceilf(" + x + ")"); break;
          case OpKind::Logistic: out = emit("1.f / (1.f + expf(-" + x + "))"); break;
          default: throw std::runtime_error("codegen: unhandled unary op");
        }
      } else {
        throw std::runtime_error(std::string("codegen: cannot fuse ") + opkind_name(op.kind));
      }
    }
  }
  c.memo.back()[key] = out;
  return out;
}

std::string CodeGen::header(const std::string& name, const Ctx& c, int extra_ptrs) const {
  std::ostringstream h;
  int np = (int)c.leaves.size() + 1 + extra_ptrs;
  h << "struct __align__(8) A_" << name << " { const void* p[" << np << "]; };\n";
  h << "extern \"C\" __global__ void __launch_bounds__(" << kThreads << ") " << name << "(const A_" << name
    << " a) {\n" << kPdlPrologue;
  for (size_t i = 0; i < c.leaves.size(); ++i) {
    const Type& t = f_.value_types[c.leaves[i]];
    h << "  const " << mtype_of(t.dtype) << "* __restrict__ L" << i << " = (const " << mtype_of(t.dtype)
      << "*)a.p[" << i << "];\n";
  }
  return h.str();
}

void CodeGen::gen_loop(const Op& root, Step* st) {
  {
    const auto& sh = root.type.shape;
    if (!sh.empty() && sh.back() % 4 == 0 && root.type.numel() > 0 &&
        (root.type.dtype == DType::F32 || root.type.dtype == DType::BF16) && gen_loop_vec4(root, st))
      return;
  }
  const std::string start_text = src_.str();
  struct Snip {
    CodeGen* g; size_t start;
    ~Snip() { g->snippets_.push_back(g->src_.str().substr(start)); }
  } snip{this, start_text.size()};
  if (root.type.numel() == 0) {
    std::string name = "k" + std::to_string(names_.size());
    // launched with programmatic dependent launch like every other kernel, so
    // it waits for its predecessor too: a later kernel's wait then covers it
    src_ << "extern \"C\" __global__ void " << name << "(const void* p) {\n" << kPdlPrologue << "}\n\n";
    names_.push_back(name);
    st->kernel = name;
    st->grid = 1;
    st->block = 32;
    return;
  }
  const auto& sh = root.type.shape;
  int r = (int)sh.size();
  Ctx c;
  c.root = root.result;
  c.idx = index_type(root, 0);
  c.memo.emplace_back();
  std::vector<std::string> coords(r);
  c.indent = 2;
  std::ostringstream pre;
  if (r > 0) {
    pre << "    " << c.idx << " r_ = i;\n";
    for (int d = r - 1; d >= 0; --d) {
      coords[d] = "c" + std::to_string(d);
      if (d == 0) pre << "    const " << c.idx << " c0 = r_;\n";
      else pre << "    const " << c.idx << " c" << d << " = r_ % " << sh[d] << "; r_ /= " << sh[d] << ";\n";
    }
  }
  // The root itself is evaluated as a cluster node: force non-materialized view.
  Val v = eval(c, root.result, coords);
  std::string name = "k" + std::to_string(names_.size());
  const char* ot = mtype_of(root.type.dtype);
  int64_t n = root.type.numel();
  src_ << header(name, c, 0);
  src_ << "  " << ot << "* __restrict__ O = (" << ot << "*)a.p[" << c.leaves.size() << "];\n";
  src_ << "  for (" << c.idx << " i = (" << c.idx << ")blockIdx.x * " << kThreads << " + threadIdx.x; i < ("
       << c.idx << ")" << n << "; i += (" << c.idx << ")gridDim.x * " << kThreads << ") {\n";
  src_ << pre.str();
  c.indent = 2;
  src_ << c.body.str();
  src_ << "    O[i] = " << store(root, v.name) << ";\n  }\n}\n\n";
  names_.push_back(name);
  st->kernel = name;
  st->leaves = c.leaves;
  st->block = kThreads;
  st->grid = std::max<int64_t>(1, std::min<int64_t>((n + kThreads - 1) / kThreads, kMaxGrid));
  int64_t bytes = n * dtype_bytes(root.type.dtype);
  for (int l : c.leaves) bytes += f_.value_types[l].numel() * dtype_bytes(f_.value_types[l].dtype);
  st->bytes_moved = bytes;
}

// Loop kernel computing 4 consecutive outputs per thread (innermost extent a
// multiple of 4, f32 output): float4 loads of contiguous leaves, uniform values
// computed once per lane group, one float4 store.  Returns false (nothing
// emitted) when an access pattern does not vectorize.
bool CodeGen::gen_loop_vec4(const Op& root, Step* st) {
  const auto& sh = root.type.shape;
  const int r = (int)sh.size();
  const int64_t n = root.type.numel();
  const int64_t q = sh[r - 1] / 4;
  Ctx c;
  c.root = root.result;
  c.idx = index_type(root, 0);
  c.memo.emplace_back();
  c.vec = true;
  c.indent = 2;
  std::vector<std::string> coords(r);
  std::ostringstream pre;
  pre << "    " << c.idx << " r_ = i;\n";
  pre << "    const " << c.idx << " cL = (r_ % " << q << ") * 4; r_ /= " << q << ";\n";
  for (int d = r - 2; d >= 0; --d) {
    coords[d] = "c" + std::to_string(d);
    if (d == 0) pre << "    const " << c.idx << " c0 = r_;\n";
    else pre << "    const " << c.idx << " c" << d << " = r_ % " << sh[d] << "; r_ /= " << sh[d] << ";\n";
  }
  std::string lanes[4];
  try {
    for (int j = 0; j < 4; ++j) {
      coords[r - 1] = kLane[j];
      lanes[j] = store(root, eval(c, root.result, coords).name);
    }
  } catch (const VecFail&) {
    return false;
  }
  const std::string start_text = src_.str();
  struct Snip {
    CodeGen* g; size_t start;
    ~Snip() { g->snippets_.push_back(g->src_.str().substr(start)); }
  } snip{this, start_text.size()};
  std::string name = "k" + std::to_string(names_.size());
  const int64_t nv = n / 4;
  const bool obf = root.type.dtype == DType::BF16;
  src_ << header(name, c, 0);
  src_ << "  " << mtype_of(root.type.dtype) << "* __restrict__ O = (" << mtype_of(root.type.dtype) << "*)a.p["
       << c.leaves.size() << "];\n";
  src_ << "  for (" << c.idx << " i = (" << c.idx << ")blockIdx.x * " << kThreads << " + threadIdx.x; i < ("
       << c.idx << ")" << nv << "; i += (" << c.idx << ")gridDim.x * " << kThreads << ") {\n";
  src_ << pre.str();
  src_ << c.body.str();
  if (obf)  // 4 bf16 in one 8-byte store
    src_ << "    *(uint2*)(O + i * 4) = make_uint2(sb_pack2(" << lanes[0] << ", " << lanes[1] << "), sb_pack2("
         << lanes[2] << ", " << lanes[3] << "));\n  }\n}\n\n";
  else
    src_ << "    *(float4*)(O + i * 4) = make_float4(" << lanes[0] << ", " << lanes[1] << ", " << lanes[2] << ", "
         << lanes[3] << ");\n  }\n}\n\n";
  names_.push_back(name);
  st->kernel = name;
  st->leaves = c.leaves;
  st->block = kThreads;
  st->grid = std::max<int64_t>(1, std::min<int64_t>((nv + kThreads - 1) / kThreads, kMaxGrid));
  int64_t bytes = n * dtype_bytes(root.type.dtype);
  for (int l : c.leaves) bytes += f_.value_types[l].numel() * dtype_bytes(f_.value_types[l].dtype);
  st->bytes_moved = bytes;
  return true;
}

// 4-wide reductions (f32).  Row mode (reduced dims trailing, R <= 4096): a
// warp per output, each lane consuming 4 consecutive elements of the innermost
// reduced dim per step.  Column mode (innermost dim kept): a thread per 4
// adjacent outputs with 4 accumulators, optionally split over the reduced
// range like the scalar column kernel.  Partial sums are combined in a fixed
// order, so results are deterministic.  Returns false (nothing emitted) when an
// access does not vectorize or the shape does not qualify.
std::string CodeGen::epilogue_code(Ctx& c, const Op& red, const Op& epi, const std::vector<std::string>& oc,
                                   int indent, std::string* val, const std::string& rv) {
  auto saved_memo = std::move(c.memo);
  const int saved_root = c.root, saved_indent = c.indent;
  const bool saved_vec = c.vec;
  std::string saved_body = c.body.str();
  c.body.str("");
  c.memo.assign(1, {});
  // the reduced value at its coordinates (unit dims read as "0", as the unit
  // reshapes between it and the epilogue root produce them) and the root's
  // coordinates: the non-unit output coordinates in order, "0" elsewhere
  const auto& xs = red.type.shape;
  std::vector<std::string> xc(xs.size()), nu;
  for (size_t d = 0; d < xs.size(); ++d) {
    xc[d] = xs[d] == 1 ? "0" : oc[d];
    if (xs[d] != 1) nu.push_back(oc[d]);
  }
  std::vector<std::string> rc;
  size_t k = 0;
  for (int64_t e : epi.type.shape) rc.push_back(e == 1 ? "0" : nu[k++]);
  c.memo[0][std::to_string(red.result) + "@" + join(xc, ",")] = Val{rv, "float"};
  c.root = epi.result;
  c.indent = indent;
  c.vec = false;
  Val v = eval(c, epi.result, rc);
  std::string code = c.body.str();
  *val = v.name;
  c.body.str(saved_body);
  c.body.seekp(0, std::ios_base::end);
  c.memo = std::move(saved_memo);
  c.root = saved_root;
  c.indent = saved_indent;
  c.vec = saved_vec;
  return code;
}

bool CodeGen::gen_reduce_vec4(const Op& root, Step* st, const Op* epi) {
  const Type& in = f_.value_types[root.operands[0]];
  const auto& ish = in.shape;
  const int r = (int)ish.size();
  auto fp = [](DType t) { return t == DType::F32 || t == DType::BF16; };
  if (r == 0 || ish[r - 1] % 4 || !fp(root.type.dtype) || !fp(in.dtype) || (epi && !fp(epi->type.dtype)))
    return false;
  // bf16 (input or stored output): row mode only (its stores are scalar)
  const bool any_bf = root.type.dtype == DType::BF16 || in.dtype == DType::BF16 ||
                      (epi && epi->type.dtype == DType::BF16);
  std::vector<int64_t> rd(root.dims.begin(), root.dims.end());
  std::sort(rd.begin(), rd.end());
  std::vector<int64_t> kd;
  for (int d = 0; d < r; ++d) if (!std::count(rd.begin(), rd.end(), d)) kd.push_back(d);
  int64_t R = 1, O = 1;
  for (auto d : rd) R *= ish[d];
  for (auto d : kd) O *= ish[d];
  bool trailing = true;
  for (size_t i = 0; i < rd.size(); ++i) if (rd[rd.size() - 1 - i] != r - 1 - (int64_t)i) trailing = false;
  const bool inner_reduced = !rd.empty() && rd.back() == r - 1;
  int mode;
  if (trailing && R <= 4096 && inner_reduced) mode = 0;
  else if (!any_bf && !epi && !trailing && !inner_reduced && !kd.empty() && kd.back() == r - 1) mode = 2;
  else return false;
  if (R == 0 || O == 0) return false;
  const char* ident = root.body == ReduceBody::Add ? "0.f"
                      : root.body == ReduceBody::Max ? "__int_as_float(0xff800000)"
                      : root.body == ReduceBody::Min ? "__int_as_float(0x7f800000)" : "1.f";
  auto combine = [&](const std::string& a, const std::string& b) {
    switch (root.body) {
      case ReduceBody::Add: return a + " + " + b;
      case ReduceBody::Max: return "fmaxf(" + a + ", " + b + ")";
      case ReduceBody::Min: return "fminf(" + a + ", " + b + ")";
      case ReduceBody::Mul: return a + " * " + b;
    }
    return a;
  };
  Ctx c;
  c.root = root.result;
  c.idx = index_type(root, 0);
  c.memo.emplace_back();
  c.vec = true;
  // coordinates: the lane coordinate "cL" is the innermost input coordinate
  // (a reduced one in row mode, a kept one in column mode)
  std::ostringstream pre, loopb;
  std::vector<std::string> oc(kd.size(), "0"), kc(rd.size(), "0");
  int64_t splits = 1, chunk = R;
  if (mode == 0) {
    if (!kd.empty()) {
      pre << "    " << c.idx << " ro_ = o;\n";
      for (int j = (int)kd.size() - 1; j >= 0; --j) {
        oc[j] = "o" + std::to_string(j);
        if (j == 0) pre << "    const " << c.idx << " o0 = ro_;\n";
        else pre << "    const " << c.idx << " o" << j << " = ro_ % " << ish[kd[j]] << "; ro_ /= " << ish[kd[j]] << ";\n";
      }
    }
    const int64_t e = ish[rd.back()];
    loopb << "      " << c.idx << " rk_ = k4 * 4;\n";
    loopb << "      const " << c.idx << " cL = rk_ % " << e << "; rk_ /= " << e << ";\n";
    for (int j = (int)rd.size() - 2; j >= 0; --j) {
      kc[j] = "q" + std::to_string(j);
      if (j == 0) loopb << "      const " << c.idx << " q0 = rk_;\n";
      else loopb << "      const " << c.idx << " q" << j << " = rk_ % " << ish[rd[j]] << "; rk_ /= " << ish[rd[j]] << ";\n";
    }
  } else {
    const int64_t e = ish[kd.back()];
    pre << "    " << c.idx << " ro_ = o4 * 4;\n";
    pre << "    const " << c.idx << " cL = ro_ % " << e << "; ro_ /= " << e << ";\n";
    for (int j = (int)kd.size() - 2; j >= 0; --j) {
      oc[j] = "o" + std::to_string(j);
      if (j == 0) pre << "    const " << c.idx << " o0 = ro_;\n";
      else pre << "    const " << c.idx << " o" << j << " = ro_ % " << ish[kd[j]] << "; ro_ /= " << ish[kd[j]] << ";\n";
    }
    loopb << "      " << c.idx << " rk_ = k;\n";
    for (int j = (int)rd.size() - 1; j >= 0; --j) {
      kc[j] = "q" + std::to_string(j);
      if (j == 0) loopb << "      const " << c.idx << " q0 = rk_;\n";
      else loopb << "      const " << c.idx << " q" << j << " = rk_ % " << ish[rd[j]] << "; rk_ /= " << ish[rd[j]] << ";\n";
    }
    // a block covers 32 float4 column groups x 8 row lanes; enough splits of
    // the reduced range for ~148 x 1536 threads, at least 32 rows per split
    const int64_t O4 = O / 4;
    const int64_t blocks_x = (O4 + 31) / 32;
    const int64_t want = (148 * 6 + blocks_x - 1) / blocks_x;
    splits = std::max<int64_t>(1, std::min<int64_t>(want, R / 32));
    chunk = (R + splits - 1) / splits;
    splits = (R + chunk - 1) / chunk;
  }
  std::string lanes[4];
  c.indent = 3;
  try {
    for (int j = 0; j < 4; ++j) {
      std::vector<std::string> ic(r);
      for (size_t q = 0; q < kd.size(); ++q) ic[kd[q]] = oc[q];
      for (size_t q = 0; q < rd.size(); ++q) ic[rd[q]] = kc[q];
      ic[r - 1] = kLane[j];
      lanes[j] = eval(c, root.operands[0], ic).name;
    }
  } catch (const VecFail&) {
    return false;
  }
  const std::string loop_code = loopb.str() + c.body.str();
  c.body.str("");
  c.vec = false;
  auto saved_memo = std::move(c.memo);
  c.memo.assign(1, {});
  c.indent = 3;
  Val init = eval(c, root.operands[1], {});
  const std::string init_code = c.body.str();
  c.memo = std::move(saved_memo);
  // final write of output o from the reduced value `acc`
  std::string epi_val, epi_code;
  if (epi) epi_code = epilogue_code(c, root, *epi, oc, 3, &epi_val);
  auto final_store = [&](const std::string& acc) {
    if (!epi) return init_code + "      O[o] = " + store(root, combine(acc, init.name)) + ";\n";
    return init_code + "      const float rv_ = " + combine(acc, init.name) + ";\n" + epi_code + "      O[o] = " +
           store(*epi, epi_val) + ";\n";
  };

  const std::string start_text = src_.str();
  struct Snip {
    CodeGen* g; size_t start;
    ~Snip() { g->snippets_.push_back(g->src_.str().substr(start)); }
  } snip{this, start_text.size()};
  std::string name = "k" + std::to_string(names_.size());
  src_ << header(name, c, mode == 2 && splits > 1 ? 1 : 0);
  {
    const char* ot = mtype_of((epi ? *epi : root).type.dtype);
    src_ << "  " << ot << "* __restrict__ O = (" << ot << "*)a.p[" << c.leaves.size() << "];\n";
  }
  if (mode == 0) {
    src_ << "  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;\n";
    src_ << "  for (" << c.idx << " o = (" << c.idx << ")blockIdx.x * " << kThreads / 32 << " + warp; o < " << O
         << "; o += (" << c.idx << ")gridDim.x * " << kThreads / 32 << ") {\n";
    src_ << pre.str();
    src_ << "    float acc = " << ident << ";\n";
    const int64_t J = (R / 4 + 31) / 32;
    if (J <= 16) {
      // unrolled lane-strided passes: every load of the row in flight at once
      src_ << "#pragma unroll\n    for (int j_ = 0; j_ < " << J << "; ++j_) {\n      const " << c.idx
           << " k4 = lane + 32 * j_;\n";
      src_ << ((R / 4) % 32 ? "      if (k4 < " + std::to_string(R / 4) + ") {\n" : std::string("      {\n"))
           << loop_code;
      for (int j = 0; j < 4; ++j) src_ << "      acc = " << combine("acc", lanes[j]) << ";\n";
      src_ << "    }}\n";
    } else {
      src_ << "    for (" << c.idx << " k4 = lane; k4 < " << R / 4 << "; k4 += 32) {\n" << loop_code;
      for (int j = 0; j < 4; ++j) src_ << "      acc = " << combine("acc", lanes[j]) << ";\n";
      src_ << "    }\n";
    }
    src_ << "    for (int s = 16; s > 0; s >>= 1) { const float y_ = __shfl_xor_sync(0xffffffffu, acc, s); acc = "
         << combine("acc", "y_") << "; }\n";
    src_ << "    if (lane == 0) {\n" << final_store("acc") << "    }\n  }\n}\n\n";
    st->grid = std::max<int64_t>(1, std::min<int64_t>((O + 7) / 8, kMaxGrid));
  } else {
    const int64_t O4 = O / 4;
    if (splits > 1) src_ << "  float* __restrict__ S = (float*)a.p[" << c.leaves.size() + 1 << "];\n";
    src_ << "  __shared__ float4 part_[8][32];\n";
    src_ << "  const int cx = threadIdx.x & 31, ry = threadIdx.x >> 5;\n";
    src_ << "  const " << c.idx << " o4 = (" << c.idx << ")blockIdx.x * 32 + cx;\n";
    src_ << "  float a0 = " << ident << ", a1 = " << ident << ", a2 = " << ident << ", a3 = " << ident << ";\n";
    src_ << "  if (o4 < " << O4 << ") {\n";
    src_ << pre.str();
    src_ << "    const " << c.idx << " k0 = (" << c.idx << ")blockIdx.y * " << chunk << ";\n";
    src_ << "    const " << c.idx << " k1 = min((" << c.idx << ")" << R << ", k0 + (" << c.idx << ")" << chunk << ");\n";
    src_ << "#pragma unroll 4\n    for (" << c.idx << " k = k0 + ry; k < k1; k += 8) {\n" << loop_code;
    for (int j = 0; j < 4; ++j) src_ << "      a" << j << " = " << combine("a" + std::to_string(j), lanes[j]) << ";\n";
    src_ << "    }\n  }\n";
    src_ << "  part_[ry][cx] = make_float4(a0, a1, a2, a3);\n  __syncthreads();\n";
    src_ << "  if (ry == 0 && o4 < " << O4 << ") {\n";
    src_ << "    for (int j = 1; j < 8; ++j) {\n      const float4 q = part_[j][cx];\n";
    src_ << "      a0 = " << combine("a0", "q.x") << "; a1 = " << combine("a1", "q.y") << "; a2 = " << combine("a2", "q.z")
         << "; a3 = " << combine("a3", "q.w") << ";\n    }\n";
    if (splits > 1) {
      src_ << "    *(float4*)(S + (" << c.idx << ")blockIdx.y * " << O << " + o4 * 4) = make_float4(a0, a1, a2, a3);\n  }\n}\n\n";
    } else {
      src_ << init_code << "    *(float4*)(O + o4 * 4) = make_float4(" << store(root, combine("a0", init.name)) << ", "
           << store(root, combine("a1", init.name)) << ", " << store(root, combine("a2", init.name)) << ", "
           << store(root, combine("a3", init.name)) << ");\n  }\n}\n\n";
    }
    st->grid = (O4 + 31) / 32;
    st->grid_y = splits;
    if (splits > 1) {
      std::string fin = name + "f";
      src_ << "struct __align__(8) A_" << fin << " { const void* p[" << c.leaves.size() + 2 << "]; };\n";
      src_ << "extern \"C\" __global__ void __launch_bounds__(" << kThreads << ") " << fin << "(const A_" << fin
           << " a) {\n" << kPdlPrologue;
      for (size_t i = 0; i < c.leaves.size(); ++i) {
        const Type& t = f_.value_types[c.leaves[i]];
        src_ << "  const " << mtype_of(t.dtype) << "* __restrict__ L" << i << " = (const " << mtype_of(t.dtype)
             << "*)a.p[" << i << "];\n";
      }
      src_ << "  float* __restrict__ O = (float*)a.p[" << c.leaves.size() << "];\n";
      src_ << "  const float* __restrict__ S = (const float*)a.p[" << c.leaves.size() + 1 << "];\n";
      // 8 float4 columns x 32 split lanes per block (lane ry takes every 32nd
      // split), then a fixed tree over the 32 lanes: deterministic
      src_ << "  __shared__ float4 part_[32][8];\n";
      src_ << "  const int cx = threadIdx.x & 7, ry = threadIdx.x >> 3;\n";
      src_ << "  const " << c.idx << " o4 = (" << c.idx << ")blockIdx.x * 8 + cx;\n";
      src_ << "  float a0 = " << ident << ", a1 = " << ident << ", a2 = " << ident << ", a3 = " << ident << ";\n";
      src_ << "  if (o4 < " << O4 << ") {\n";
      src_ << "#pragma unroll 4\n    for (" << c.idx << " s = ry; s < " << splits << "; s += 32) {\n";
      src_ << "      const float4 q = *(const float4*)(S + s * " << O << " + o4 * 4);\n";
      src_ << "      a0 = " << combine("a0", "q.x") << "; a1 = " << combine("a1", "q.y") << "; a2 = "
           << combine("a2", "q.z") << "; a3 = " << combine("a3", "q.w") << ";\n    }\n  }\n";
      src_ << "  part_[ry][cx] = make_float4(a0, a1, a2, a3);\n  __syncthreads();\n";
      src_ << "  for (int w = 16; w > 0; w >>= 1) {\n    if (ry < w) {\n";
      src_ << "      const float4 p = part_[ry][cx], q = part_[ry + w][cx];\n";
      src_ << "      part_[ry][cx] = make_float4(" << combine("p.x", "q.x") << ", " << combine("p.y", "q.y") << ", "
           << combine("p.z", "q.z") << ", " << combine("p.w", "q.w") << ");\n    }\n    __syncthreads();\n  }\n";
      src_ << "  if (ry == 0 && o4 < " << O4 << ") {\n";
      src_ << "    const float4 q = part_[0][cx];\n    a0 = q.x; a1 = q.y; a2 = q.z; a3 = q.w;\n";
      src_ << init_code << "    *(float4*)(O + o4 * 4) = make_float4(" << store(root, combine("a0", init.name)) << ", "
           << store(root, combine("a1", init.name)) << ", " << store(root, combine("a2", init.name)) << ", "
           << store(root, combine("a3", init.name)) << ");\n  }\n}\n\n";
      names_.push_back(fin);
      st->finish_kernel = fin;
      st->finish_grid = (O4 + 7) / 8;
      st->splits = splits;
      st->scratch_elems = splits * O;
    }
  }
  names_.push_back(name);
  st->kernel = name;
  st->leaves = c.leaves;
  st->block = kThreads;
  int64_t bytes = O * 4;
  for (int l : c.leaves) bytes += f_.value_types[l].numel() * dtype_bytes(f_.value_types[l].dtype);
  st->bytes_moved = bytes;
  return true;
}

void CodeGen::gen_reduce(const Op& root, Step* st, const Op* epi) {
  if (gen_reduce_vec4(root, st, epi)) return;
  const std::string start_text = src_.str();
  struct Snip {
    CodeGen* g; size_t start;
    ~Snip() { g->snippets_.push_back(g->src_.str().substr(start)); }
  } snip{this, start_text.size()};
  const Type& in = f_.value_types[root.operands[0]];
  const auto& ish = in.shape;
  int r = (int)ish.size();
  std::vector<int64_t> rd(root.dims.begin(), root.dims.end());
  std::sort(rd.begin(), rd.end());
  std::vector<int64_t> kd;  // kept dims
  for (int d = 0; d < r; ++d) if (!std::count(rd.begin(), rd.end(), d)) kd.push_back(d);
  int64_t R = 1, O = 1;
  for (auto d : rd) R *= ish[d];
  for (auto d : kd) O *= ish[d];
  bool trailing = true;
  for (size_t i = 0; i < rd.size(); ++i) if (rd[rd.size() - 1 - i] != r - 1 - (int64_t)i) trailing = false;
  const char* ident = root.body == ReduceBody::Add ? "0.f"
                      : root.body == ReduceBody::Max ? "__int_as_float(0xff800000)"
                      : root.body == ReduceBody::Min ? "__int_as_float(0x7f800000)" : "1.f";
  auto combine = [&](const std::string& a, const std::string& b) {
    switch (root.body) {
      case ReduceBody::Add: return a + " + " + b;
      case ReduceBody::Max: return "fmaxf(" + a + ", " + b + ")";
      case ReduceBody::Min: return "fminf(" + a + ", " + b + ")";
      case ReduceBody::Mul: return a + " * " + b;
    }
    return a;
  };
  // bf16 reductions accumulate in f32 and round the result once
  auto fp = [](DType t) { return t == DType::F32 || t == DType::BF16; };
  if (!fp(root.type.dtype) || !fp(in.dtype) || (epi && !fp(epi->type.dtype)))
    throw std::runtime_error("reduce: only f32 and bf16 reductions are supported");

  Ctx c;
  c.root = root.result;
  c.idx = index_type(root, 0);
  c.memo.emplace_back();
  std::string name = "k" + std::to_string(names_.size());
  std::ostringstream body;  // assembled kernel body after leaves are known
  auto out_coords = [&](std::ostringstream& os, const std::string& oi, std::vector<std::string>& oc,
                        const std::string& ind) {
    oc.assign(kd.size(), "0");
    if (kd.empty()) return;
    os << ind << c.idx << " ro_ = " << oi << ";\n";
    for (int j = (int)kd.size() - 1; j >= 0; --j) {
      oc[j] = "o" + std::to_string(j);
      if (j == 0) os << ind << "const " << c.idx << " o0 = ro_;\n";
      else os << ind << "const " << c.idx << " o" << j << " = ro_ % " << ish[kd[j]] << "; ro_ /= " << ish[kd[j]] << ";\n";
    }
  };
  auto red_coords = [&](std::ostringstream& os, std::vector<std::string>& kc, const std::string& ind) {
    kc.assign(rd.size(), "0");
    os << ind << c.idx << " rk_ = k;\n";
    for (int j = (int)rd.size() - 1; j >= 0; --j) {
      kc[j] = "q" + std::to_string(j);
      if (j == 0) os << ind << "const " << c.idx << " q0 = rk_;\n";
      else os << ind << "const " << c.idx << " q" << j << " = rk_ % " << ish[rd[j]] << "; rk_ /= " << ish[rd[j]] << ";\n";
    }
  };
  auto merged = [&](const std::vector<std::string>& oc, const std::vector<std::string>& kc) {
    std::vector<std::string> ic(r);
    for (size_t j = 0; j < kd.size(); ++j) ic[kd[j]] = oc[j];
    for (size_t j = 0; j < rd.size(); ++j) ic[rd[j]] = kc[j];
    return ic;
  };

  std::ostringstream pre, loopb, post;
  std::vector<std::string> oc, kc;
  int64_t splits = 1, chunk = R;
  int mode;  // 0 warp/row, 1 block/row, 2 column
  if (trailing && R <= 4096) mode = 0;
  else if (trailing) mode = 1;
  else mode = 2;
  if (mode == 1 && O < 2 * 148 && R >= 2 * 8192) {
    // few long rows (a merged full reduction): blocks split each row, a
    // finish kernel combines the partials in split order
    splits = std::min<int64_t>((148 * 4 + O - 1) / O, R / 4096);
    splits = std::max<int64_t>(splits, 1);
    chunk = (R + splits - 1) / splits;
    splits = (R + chunk - 1) / chunk;
  }
  if (mode == 2) {
    int64_t target = 148 * 2048;
    if (O < target && R >= 64) {
      splits = std::min<int64_t>((target + O - 1) / O, R / 8);
      splits = std::max<int64_t>(splits, 1);
      chunk = (R + splits - 1) / splits;
      splits = (R + chunk - 1) / chunk;
    }
  }
  // body of the accumulation loop (input expression at merged coords)
  c.indent = 3;
  red_coords(loopb, kc, "      ");
  c.body.str("");
  out_coords(pre, mode == 2 ? "o" : "o", oc, "    ");
  Val v = eval(c, root.operands[0], merged(oc, kc));
  std::string loop_code = loopb.str() + c.body.str();
  // init value (scalar expression), evaluated in its own scope
  c.body.str("");
  auto saved_memo = std::move(c.memo);
  c.memo.assign(1, {});
  c.indent = 3;
  Val init = eval(c, root.operands[1], {});
  std::string init_code = c.body.str();
  c.memo = std::move(saved_memo);
  // final write of output o from the reduced value `acc`
  std::string epi_val, epi_code;
  if (epi) epi_code = epilogue_code(c, root, *epi, oc, 3, &epi_val);
  auto final_store = [&](const std::string& acc) {
    if (!epi) return init_code + "      O[o] = " + store(root, combine(acc, init.name)) + ";\n";
    return init_code + "      const float rv_ = " + combine(acc, init.name) + ";\n" + epi_code + "      O[o] = " +
           store(*epi, epi_val) + ";\n";
  };

  src_ << header(name, c, splits > 1 ? 1 : 0);
  {
    const char* ot = mtype_of((epi ? *epi : root).type.dtype);
    src_ << "  " << ot << "* __restrict__ O = (" << ot << "*)a.p[" << c.leaves.size() << "];\n";
  }
  if (mode == 0) {
    src_ << "  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;\n";
    src_ << "  for (" << c.idx << " o = (" << c.idx << ")blockIdx.x * " << kThreads / 32 << " + warp; o < " << O
         << "; o += (" << c.idx << ")gridDim.x * " << kThreads / 32 << ") {\n";
    src_ << pre.str();
    src_ << "    float acc = " << ident << ";\n";
    src_ << "    for (" << c.idx << " k = lane; k < " << R << "; k += 32) {\n" << loop_code;
    src_ << "      acc = " << combine("acc", v.name) << ";\n    }\n";
    src_ << "    for (int s = 16; s > 0; s >>= 1) { const float y_ = __shfl_xor_sync(0xffffffffu, acc, s); acc = "
         << combine("acc", "y_") << "; }\n";
    src_ << "    if (lane == 0) {\n" << final_store("acc") << "    }\n  }\n}\n\n";
    st->grid = std::max<int64_t>(1, std::min<int64_t>((O + 7) / 8, kMaxGrid));
  } else if (mode == 1) {
    if (splits > 1) src_ << "  float* __restrict__ S = (float*)a.p[" << c.leaves.size() + 1 << "];\n";
    src_ << "  __shared__ float red_[" << kThreads / 32 << "];\n";
    src_ << "  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;\n";
    src_ << "  const " << c.idx << " k0 = (" << c.idx << ")blockIdx.y * " << chunk << ";\n";
    src_ << "  const " << c.idx << " k1 = min((" << c.idx << ")" << R << ", k0 + (" << c.idx << ")" << chunk << ");\n";
    src_ << "  for (" << c.idx << " o = blockIdx.x; o < " << O << "; o += gridDim.x) {\n";
    src_ << pre.str();
    src_ << "    float acc = " << ident << ";\n";
    src_ << "#pragma unroll 4\n    for (" << c.idx << " k = k0 + threadIdx.x; k < k1; k += " << kThreads << ") {\n" << loop_code;
    src_ << "      acc = " << combine("acc", v.name) << ";\n    }\n";
    src_ << "    for (int s = 16; s > 0; s >>= 1) { const float y_ = __shfl_xor_sync(0xffffffffu, acc, s); acc = "
         << combine("acc", "y_") << "; }\n";
    src_ << "    if (lane == 0) red_[warp] = acc;\n    __syncthreads();\n";
    src_ << "    if (warp == 0) {\n      acc = lane < " << kThreads / 32 << " ? red_[lane] : " << ident << ";\n";
    src_ << "      for (int s = 16; s > 0; s >>= 1) { const float y_ = __shfl_xor_sync(0xffffffffu, acc, s); acc = "
         << combine("acc", "y_") << "; }\n";
    if (splits > 1)
      src_ << "      if (lane == 0) S[(" << c.idx << ")blockIdx.y * " << O << " + o] = acc;\n    }\n";
    else
      src_ << "      if (lane == 0) {\n" << final_store("acc") << "      }\n    }\n";
    src_ << "    __syncthreads();\n  }\n}\n\n";
    st->grid = std::max<int64_t>(1, std::min<int64_t>(O, kMaxGrid));
    st->grid_y = splits;
  } else {
    if (splits > 1) src_ << "  float* __restrict__ S = (float*)a.p[" << c.leaves.size() + 1 << "];\n";
    src_ << "  for (" << c.idx << " o = (" << c.idx << ")blockIdx.x * " << kThreads << " + threadIdx.x; o < " << O
         << "; o += (" << c.idx << ")gridDim.x * " << kThreads << ") {\n";
    src_ << pre.str();
    src_ << "    float acc = " << ident << ";\n";
    src_ << "    const " << c.idx << " k0 = (" << c.idx << ")blockIdx.y * " << chunk << ";\n";
    src_ << "    const " << c.idx << " k1 = min((" << c.idx << ")" << R << ", k0 + (" << c.idx << ")" << chunk << ");\n";
    src_ << "#pragma unroll 4\n    for (" << c.idx << " k = k0; k < k1; ++k) {\n" << loop_code;
    src_ << "      acc = " << combine("acc", v.name) << ";\n    }\n";
    if (splits > 1) {
      src_ << "    S[(" << c.idx << ")blockIdx.y * " << O << " + o] = acc;\n  }\n}\n\n";
    } else {
      src_ << "    {\n" << final_store("acc") << "    }\n  }\n}\n\n";
    }
    st->grid = std::max<int64_t>(1, std::min<int64_t>((O + kThreads - 1) / kThreads, kMaxGrid));
    st->grid_y = splits;
  }
  if (splits > 1) {
    {
      std::string fin = name + "f";
      src_ << "struct __align__(8) A_" << fin << " { const void* p[" << c.leaves.size() + 2 << "]; };\n";
      src_ << "extern \"C\" __global__ void __launch_bounds__(" << kThreads << ") " << fin << "(const A_" << fin
           << " a) {\n" << kPdlPrologue;
      for (size_t i = 0; i < c.leaves.size(); ++i) {
        const Type& t = f_.value_types[c.leaves[i]];
        src_ << "  const " << mtype_of(t.dtype) << "* __restrict__ L" << i << " = (const " << mtype_of(t.dtype)
             << "*)a.p[" << i << "];\n";
      }
      {
        const char* ot = mtype_of((epi ? *epi : root).type.dtype);
        src_ << "  " << ot << "* __restrict__ O = (" << ot << "*)a.p[" << c.leaves.size() << "];\n";
      }
      src_ << "  const float* __restrict__ S = (const float*)a.p[" << c.leaves.size() + 1 << "];\n";
      const bool block_per_output = O <= 2 * 148;
      if (block_per_output) {
        // one block per output: threads take the partials of a strided
        // subset of splits, then a fixed shuffle/shared-memory tree
        src_ << "  __shared__ float red_[" << kThreads / 32 << "];\n";
        src_ << "  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;\n";
        src_ << "  for (" << c.idx << " o = blockIdx.x; o < " << O << "; o += gridDim.x) {\n";
        if (epi) src_ << pre.str();
        src_ << "    float acc = " << ident << ";\n";
        src_ << "#pragma unroll 4\n    for (" << c.idx << " s = threadIdx.x; s < " << splits << "; s += " << kThreads
             << ") acc = " << combine("acc", "S[s * " + std::to_string(O) + " + o]") << ";\n";
        src_ << "    for (int s = 16; s > 0; s >>= 1) { const float y_ = __shfl_xor_sync(0xffffffffu, acc, s); acc = "
             << combine("acc", "y_") << "; }\n";
        src_ << "    if (lane == 0) red_[warp] = acc;\n    __syncthreads();\n";
        src_ << "    if (warp == 0) {\n      acc = lane < " << kThreads / 32 << " ? red_[lane] : " << ident << ";\n";
        src_ << "      for (int s = 16; s > 0; s >>= 1) { const float y_ = __shfl_xor_sync(0xffffffffu, acc, s); acc = "
             << combine("acc", "y_") << "; }\n";
        src_ << "      if (lane == 0) {\n" << final_store("acc") << "      }\n    }\n    __syncthreads();\n  }\n}\n\n";
      } else {
        src_ << "  for (" << c.idx << " o = (" << c.idx << ")blockIdx.x * " << kThreads << " + threadIdx.x; o < " << O
             << "; o += (" << c.idx << ")gridDim.x * " << kThreads << ") {\n";
        if (epi) src_ << pre.str();
        src_ << "    float acc = " << ident << ";\n";
        src_ << "#pragma unroll 4\n    for (" << c.idx << " s = 0; s < " << splits << "; ++s) acc = "
             << combine("acc", "S[s * " + std::to_string(O) + " + o]") << ";\n";
        src_ << "    {\n" << final_store("acc") << "    }\n  }\n}\n\n";
      }
      names_.push_back(fin);
      st->finish_kernel = fin;
      st->finish_grid = block_per_output ? O : std::max<int64_t>(1, std::min<int64_t>((O + kThreads - 1) / kThreads, kMaxGrid));
      st->splits = splits;
      st->scratch_elems = splits * O;
    }
  }
  names_.push_back(name);
  st->kernel = name;
  st->leaves = c.leaves;
  st->block = kThreads;
  int64_t bytes = O * 4;
  for (int l : c.leaves) bytes += f_.value_types[l].numel() * dtype_bytes(f_.value_types[l].dtype);
  st->bytes_moved = bytes;
}

std::string CodeGen::prelude() {
  return "// generated by sheaf_b200 for sm_100a\n"
         "__device__ __forceinline__ float sb_rna_tf32(float x) {\n"
         "  unsigned u;\n"
         "  asm(\"cvt.rna.tf32.f32 %0, %1;\" : \"=r\"(u) : \"f\"(x));\n"
         "  return __uint_as_float(u);\n"
         "}\n"
         "// bf16 <-> f32: bf16 is the upper half of an f32; f32 -> bf16 rounds to\n"
         "// nearest even (cvt.rn.bf16.f32)\n"
         "__device__ __forceinline__ float sb_bf16_ld(unsigned short h) { return __uint_as_float((unsigned)h << 16); }\n"
         "__device__ __forceinline__ unsigned short sb_bf16_bits(float x) {\n"
         "  unsigned short h;\n"
         "  asm(\"cvt.rn.bf16.f32 %0, %1;\" : \"=h\"(h) : \"f\"(x));\n"
         "  return h;\n"
         "}\n"
         "__device__ __forceinline__ float sb_bf16_rn(float x) { return sb_bf16_ld(sb_bf16_bits(x)); }\n"
         "__device__ __forceinline__ float4 sb_bf16x4(uint2 u) {\n"
         "  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),\n"
         "                     __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));\n"
         "}\n"
         "__device__ __forceinline__ unsigned sb_pack2(unsigned short lo, unsigned short hi) {\n"
         "  return (unsigned)lo | ((unsigned)hi << 16);\n"
         "}\n";
}

bool CodeGen::gen_row_group(const std::vector<RowMember>& ms, int64_t R, int64_t C, Step* st) {
  // each lane owns J float4 groups of a row (chunk j: columns
  // (lane + 32 j) * 4 .. +3); every member's row values stay in registers
  if (ms.size() < 2 || R <= 0 || C % 128 || C / 128 > 8) return false;
  const int J = (int)(C / 128);
  Ctx c;
  c.idx = index_type(*ms[0].root, R * C);
  c.memo.assign(1, {});
  c.vec = true;
  c.indent = 2;
  std::vector<int> outs;
  std::vector<int> shadows;  // values whose operand shadows this kernel writes (X0, X1, ...)
  std::ostringstream rows;  // before the row loop: lane columns, column accumulators
  for (int j = 0; j < J; ++j)
    rows << "  const " << c.idx << " cL" << j << " = (lane + " << 32 * j << ") * 4;\n";
  // column reductions (kind 3): output index, reduce op, accumulator names
  struct ColRed {
    int out;
    const Op* op;
    std::vector<std::string> acc;  // J x 4, chunk-major
    std::string init_code, init_val;
  };
  std::vector<ColRed> cols;
  auto body_op = [](const Op& r) {
    return std::function<std::string(const std::string&, const std::string&)>(
        [&r](const std::string& a, const std::string& b) {
          switch (r.body) {
            case ReduceBody::Add: return a + " + " + b;
            case ReduceBody::Max: return "fmaxf(" + a + ", " + b + ")";
            case ReduceBody::Min: return "fminf(" + a + ", " + b + ")";
            case ReduceBody::Mul: return a + " * " + b;
          }
          return a;
        });
  };
  auto ident_of = [](const Op& r) {
    return std::string(r.body == ReduceBody::Add ? "0.f"
                       : r.body == ReduceBody::Max ? "__int_as_float(0xff800000)"
                       : r.body == ReduceBody::Min ? "__int_as_float(0x7f800000)" : "1.f");
  };
  // coordinates of a shape whose leading dims hold the row index `row`
  // (innermost dim excluded when `full`); declared once per row shape, so
  // members of the same shape share loads and subexpressions
  std::map<std::vector<int64_t>, std::vector<std::string>> coord_of;
  auto row_coords = [&](const std::vector<int64_t>& sh, bool full, const std::string&) {
    std::vector<int64_t> key(sh.begin(), sh.end() - (full ? 1 : 0));
    auto it = coord_of.find(key);
    if (it != coord_of.end()) {
      std::vector<std::string> co = it->second;
      if (full) co.push_back("0");
      return co;
    }
    const std::string tag = "r" + std::to_string(coord_of.size()) + "_";
    const int n = (int)key.size();
    std::vector<std::string> co(sh.size(), "0");
    c.body << "    " << c.idx << " " << tag << "_ = row;\n";
    for (int d = n - 1; d >= 0; --d) {
      if (sh[d] == 1) continue;
      co[d] = tag + std::to_string(d);
      c.body << "    const " << c.idx << " " << co[d] << " = " << tag << "_ % " << sh[d] << "; " << tag << "_ /= "
             << sh[d] << ";\n";
    }
    coord_of[key] = std::vector<std::string>(co.begin(), co.begin() + n);
    return co;
  };
  auto reg = [&](const std::string& expr) {
    const std::string n = fresh(c, "g");
    c.body << "    const float " << n << " = " << expr << ";\n";
    return Val{n, "float"};
  };
  try {
    for (size_t mi = 0; mi < ms.size(); ++mi) {
      const RowMember& m = ms[mi];
      const Op& root = *m.root;
      const Op& out_op = m.epi ? *m.epi : root;
      const int out_v = out_op.result;
      // bf16 outputs: the registers hold the bf16-rounded f32 value (what
      // later members read), the stores write its 16 bits
      const bool bf = out_op.type.dtype == DType::BF16;
      if (out_op.type.dtype != DType::F32 && !bf) return false;
      if (bf && m.kind == 3) return false;
      auto held = [&](const Op& o, const std::string& e) { return bf ? "sb_bf16_rn(" + e + ")" : store(o, e); };
      const std::string W = "O" + std::to_string(outs.size());
      outs.push_back(out_v);
      const std::string tag = "m" + std::to_string(mi) + "r";
      c.indent = 2;
      if (m.kind == 0) {
        const auto& sh = root.type.shape;
        if (sh.empty() || sh.back() != C) return false;
        std::vector<std::string> co = row_coords(sh, true, tag);
        c.root = root.result;
        for (int j = 0; j < J; ++j) {
          const std::string b = "cL" + std::to_string(j);
          std::string g[4];
          for (int k = 0; k < 4; ++k) {
            co.back() = lane_coord(b, k);
            const Val v = reg(held(root, eval(c, root.result, co).name));
            // later members see the stored (possibly TF32-rounded) value
            c.memo[0][std::to_string(root.result) + "@" + join(co, ",")] = v;
            c.regs[std::to_string(out_v) + "@" + b + ":" + std::to_string(k)] = v;
            g[k] = v.name;
          }
          if (bf)
            c.body << "    *(uint2*)(" << W << " + row * " << C << " + " << b << ") = make_uint2(sb_pack2(sb_bf16_bits("
                   << g[0] << "), sb_bf16_bits(" << g[1] << ")), sb_pack2(sb_bf16_bits(" << g[2] << "), sb_bf16_bits("
                   << g[3] << ")));\n";
          else
            c.body << "    *(float4*)(" << W << " + row * " << C << " + " << b << ") = make_float4(" << g[0] << ", "
                   << g[1] << ", " << g[2] << ", " << g[3] << ");\n";
          auto sv = shadow_vals_.find(out_v);
          if (sv != shadow_vals_.end()) {
            // the operand shadow of the same four values
            auto it = std::find(shadows.begin(), shadows.end(), out_v);
            const int xi = (int)(it - shadows.begin());
            if (it == shadows.end()) shadows.push_back(out_v);
            const std::string X = "X" + std::to_string(xi);
            if (sv->second == DType::BF16)
              c.body << "    *(uint2*)(" << X << " + row * " << C << " + " << b << ") = make_uint2(sb_pack2(sb_bf16_bits("
                     << g[0] << "), sb_bf16_bits(" << g[1] << ")), sb_pack2(sb_bf16_bits(" << g[2]
                     << "), sb_bf16_bits(" << g[3] << ")));\n";
            else
              c.body << "    *(float4*)(" << X << " + row * " << C << " + " << b << ") = make_float4(sb_rna_tf32("
                     << g[0] << "), sb_rna_tf32(" << g[1] << "), sb_rna_tf32(" << g[2] << "), sb_rna_tf32(" << g[3]
                     << "));\n";
          }
        }
        c.reg_kind[out_v] = 0;
      } else if (m.kind == 1) {
        if (root.type.numel() != R) return false;
        std::vector<std::string> co = row_coords(root.type.shape, false, tag);
        c.root = root.result;
        const Val v = reg(held(root, eval(c, root.result, co).name));
        c.memo[0][std::to_string(root.result) + "@" + join(co, ",")] = v;
        c.body << "    if (lane == 0) " << W << "[row] = " << (bf ? "sb_bf16_bits(" + v.name + ")" : v.name) << ";\n";
        c.regs[std::to_string(out_v) + "@row"] = v;
        c.reg_kind[out_v] = 1;
      } else if (m.kind == 3) {
        // reduction over all rows: each lane accumulates its columns over the
        // rows its warp visits; the block and the finish kernel combine the
        // lanes' partials in a fixed order after the row loop
        const Type& in = f_.value_types[root.operands[0]];
        const auto& ish = in.shape;
        const int r = (int)ish.size();
        if (r < 2 || ish.back() != C || in.numel() != R * C || root.type.numel() != C ||
            root.type.dtype != DType::F32 || in.dtype != DType::F32 || (int)root.dims.size() != r - 1)
          return false;
        for (int d = 0; d + 1 < r; ++d)
          if (root.dims[d] != d) return false;
        auto combine = body_op(root);
        std::vector<std::string> co = row_coords(ish, true, tag);
        c.root = root.result;
        ColRed cr;
        cr.out = (int)outs.size() - 1;
        cr.op = &root;
        for (int j = 0; j < J; ++j)
          for (int k = 0; k < 4; ++k) {
            co.back() = lane_coord("cL" + std::to_string(j), k);
            const std::string v = eval(c, root.operands[0], co).name;
            const std::string a = "ca" + std::to_string(cols.size()) + "_" + std::to_string(4 * j + k);
            c.body << "    " << a << " = " << combine(a, v) << ";\n";
            cr.acc.push_back(a);
            rows << "  float " << a << " = " << ident_of(root) << ";\n";
          }
        const bool saved_vec = c.vec;
        c.vec = false;
        const std::string saved_body = c.body.str();
        c.body.str("");
        c.body.clear();
        auto saved_memo = std::move(c.memo);
        c.memo.assign(1, {});
        cr.init_val = eval(c, root.operands[1], {}).name;
        cr.init_code = c.body.str();
        c.memo = std::move(saved_memo);
        c.body.str(saved_body);
        c.body.seekp(0, std::ios_base::end);
        c.vec = saved_vec;
        cols.push_back(cr);
      } else {
        const Type& in = f_.value_types[root.operands[0]];
        const auto& ish = in.shape;
        const int r = (int)ish.size();
        // f32 accumulation of f32 or bf16 rows (a bf16 result is rounded once)
        if (r == 0 || ish.back() != C || root.dims.size() != 1 || root.dims[0] != r - 1 ||
            (root.type.dtype != DType::F32 && root.type.dtype != DType::BF16) ||
            (in.dtype != DType::F32 && in.dtype != DType::BF16) || root.type.numel() != R)
          return false;
        const char* ident = root.body == ReduceBody::Add ? "0.f"
                            : root.body == ReduceBody::Max ? "__int_as_float(0xff800000)"
                            : root.body == ReduceBody::Min ? "__int_as_float(0x7f800000)" : "1.f";
        auto combine = [&](const std::string& a, const std::string& b) {
          switch (root.body) {
            case ReduceBody::Add: return a + " + " + b;
            case ReduceBody::Max: return "fmaxf(" + a + ", " + b + ")";
            case ReduceBody::Min: return "fminf(" + a + ", " + b + ")";
            case ReduceBody::Mul: return a + " * " + b;
          }
          return a;
        };
        std::vector<std::string> oc = row_coords(root.type.shape, false, tag);
        std::vector<std::string> ic(r);
        for (int d = 0; d + 1 < r; ++d) ic[d] = oc[d];
        c.root = root.result;
        // per lane in the order of the 4-wide row reduction kernel (chunk by
        // chunk, x y z w), then the xor tree: every lane holds the total
        const std::string acc = fresh(c, "acc");
        c.body << "    float " << acc << " = " << ident << ";\n";
        for (int j = 0; j < J; ++j) {
          std::string lv[4];
          for (int k = 0; k < 4; ++k) {
            ic[r - 1] = lane_coord("cL" + std::to_string(j), k);
            lv[k] = eval(c, root.operands[0], ic).name;
          }
          for (int k = 0; k < 4; ++k) c.body << "    " << acc << " = " << combine(acc, lv[k]) << ";\n";
        }
        c.body << "    for (int s = 16; s > 0; s >>= 1) { const float y_ = __shfl_xor_sync(0xffffffffu, " << acc
               << ", s); " << acc << " = " << combine(acc, "y_") << "; }\n";
        const bool saved_vec = c.vec;
        c.vec = false;
        const Val init = eval(c, root.operands[1], {});
        const bool bf_red = root.type.dtype == DType::BF16;
        const Val rv = reg(bf_red ? "sb_bf16_rn(" + combine(acc, init.name) + ")" : combine(acc, init.name));
        Val out = rv;
        if (m.epi) {
          std::string ev;
          const std::string code = epilogue_code(c, root, *m.epi, oc, 2, &ev, rv.name);
          c.body << code;
          out = reg(held(*m.epi, ev));
        } else {
          out = reg(held(root, rv.name));
        }
        c.vec = saved_vec;
        c.body << "    if (lane == 0) " << W << "[row] = " << (bf ? "sb_bf16_bits(" + out.name + ")" : out.name)
               << ";\n";
        c.regs[std::to_string(out_v) + "@row"] = out;
        c.reg_kind[out_v] = 1;
      }
    }
  } catch (const VecFail&) {
    return false;
  }
  const std::string start_text = src_.str();
  struct Snip {
    CodeGen* g; size_t start;
    ~Snip() { g->snippets_.push_back(g->src_.str().substr(start)); }
  } snip{this, start_text.size()};
  std::string name = "k" + std::to_string(names_.size());
  // with column reductions the grid is one full wave (8 blocks per SM), so
  // the per-block partials stay few while every warp slot is used
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>((R + 7) / 8, cols.empty() ? kMaxGrid : 148 * 8));
  const size_t np = c.leaves.size() + outs.size();
  src_ << header(name, c, (int)outs.size() - 1 + (cols.empty() ? 0 : 1) + (int)shadows.size());
  for (size_t j = 0; j < outs.size(); ++j) {
    const char* t = f_.value_types[outs[j]].dtype == DType::BF16 ? "unsigned short" : "float";
    src_ << "  " << t << "* __restrict__ O" << j << " = (" << t << "*)a.p[" << c.leaves.size() + j << "];\n";
  }
  for (size_t k = 0; k < shadows.size(); ++k) {
    const char* t = shadow_vals_.at(shadows[k]) == DType::BF16 ? "unsigned short" : "float";
    src_ << "  " << t << "* __restrict__ X" << k << " = (" << t << "*)a.p[" << np + (cols.empty() ? 0 : 1) + k
         << "];\n";
  }
  src_ << "  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;\n";
  src_ << rows.str();
  src_ << "  for (" << c.idx << " row = (" << c.idx << ")blockIdx.x * " << kThreads / 32 << " + warp; row < " << R
       << "; row += (" << c.idx << ")gridDim.x * " << kThreads / 32 << ") {\n";
  src_ << c.body.str() << "  }\n";
  if (!cols.empty()) {
    // per block: the 8 warps' lane partials, combined in warp order
    src_ << "  float* __restrict__ S = (float*)a.p[" << np << "];\n";
    src_ << "  __shared__ float cs_[" << kThreads / 32 << "][" << C << "];\n";
    for (size_t q = 0; q < cols.size(); ++q) {
      auto combine = body_op(*cols[q].op);
      for (int j = 0; j < J; ++j)
        for (int k = 0; k < 4; ++k)
          src_ << "  cs_[warp][cL" << j << " + " << k << "] = " << cols[q].acc[4 * j + k] << ";\n";
      src_ << "  __syncthreads();\n";
      src_ << "  for (int c_ = threadIdx.x; c_ < " << C << "; c_ += " << kThreads << ") {\n";
      src_ << "    float v_ = cs_[0][c_];\n";
      src_ << "    for (int w_ = 1; w_ < " << kThreads / 32 << "; ++w_) v_ = " << combine("v_", "cs_[w_][c_]") << ";\n";
      src_ << "    S[" << q * grid * C << " + (" << c.idx << ")blockIdx.x * " << C << " + c_] = v_;\n  }\n";
      src_ << "  __syncthreads();\n";
    }
  }
  src_ << "}\n\n";
  names_.push_back(name);
  st->kernel = name;
  st->leaves = c.leaves;
  st->root = outs[0];
  st->extra_roots.assign(outs.begin() + 1, outs.end());
  st->shadow_values = shadows;
  st->block = kThreads;
  st->grid = grid;
  if (!cols.empty()) {
    // finish: 8 columns x 32 block lanes per block, a fixed tree over the lanes
    const std::string fin = name + "f";
    src_ << "struct __align__(8) A_" << fin << " { const void* p[" << np + 1 << "]; };\n";
    src_ << "extern \"C\" __global__ void __launch_bounds__(" << kThreads << ") " << fin << "(const A_" << fin
         << " a) {\n" << kPdlPrologue;
    for (size_t i = 0; i < c.leaves.size(); ++i) {
      const Type& t = f_.value_types[c.leaves[i]];
      src_ << "  const " << mtype_of(t.dtype) << "* __restrict__ L" << i << " = (const " << mtype_of(t.dtype)
           << "*)a.p[" << i << "];\n";
    }
    src_ << "  const float* __restrict__ S = (const float*)a.p[" << np << "];\n";
    src_ << "  __shared__ float part_[32][8];\n";
    src_ << "  const int cx = threadIdx.x & 7, ry = threadIdx.x >> 3;\n";
    src_ << "  const int col = blockIdx.x * 8 + cx;\n";
    for (size_t q = 0; q < cols.size(); ++q) {
      auto combine = body_op(*cols[q].op);
      src_ << "  {\n    float v_ = " << ident_of(*cols[q].op) << ";\n";
      // a trip count known at compile time (ceil(grid / 32)): the loop is
      // unrolled and all of a thread's partial loads are in flight together
      src_ << "    if (col < " << C << ") {\n#pragma unroll\n      for (int i_ = 0; i_ < " << (grid + 31) / 32
           << "; ++i_) {\n        const int b_ = ry + 32 * i_;\n        if (b_ < " << grid << ") v_ = "
           << combine("v_", "S[" + std::to_string(q * grid * C) + " + b_ * " + std::to_string(C) + " + col]")
           << ";\n      }\n    }\n";
      src_ << "    part_[ry][cx] = v_;\n    __syncthreads();\n";
      src_ << "    for (int w_ = 16; w_ > 0; w_ >>= 1) {\n      if (ry < w_) part_[ry][cx] = "
           << combine("part_[ry][cx]", "part_[ry + w_][cx]") << ";\n      __syncthreads();\n    }\n";
      src_ << "    if (ry == 0 && col < " << C << ") {\n" << cols[q].init_code << "      ((float*)a.p["
           << c.leaves.size() + cols[q].out << "])[col] = " << store(*cols[q].op, combine("part_[0][cx]", cols[q].init_val))
           << ";\n    }\n    __syncthreads();\n  }\n";
    }
    src_ << "}\n\n";
    names_.push_back(fin);
    st->finish_kernel = fin;
    st->finish_grid = (C + 7) / 8;
    st->splits = grid;
    st->scratch_elems = (int64_t)cols.size() * grid * C;
    // plain column sums can also be finished by the batched kernel, which adds
    // in the same order (block partials by ry then the 32-lane tree, + 0)
    bool plain = true;
    for (const ColRed& cr : cols)
      plain = plain && cr.op->body == ReduceBody::Add && cr.init_code.empty() &&
              cr.init_val == "__int_as_float(0x00000000)" && store(*cr.op, "x_") == "x_" &&
              cr.op->type.dtype == DType::F32;
    if (plain)
      for (size_t q = 0; q < cols.size(); ++q) st->col_finish.push_back({cols[q].out, (int64_t)q * grid * C});
    st->col_C = C;
  }
  st->elements = R * C;
  int64_t bytes = 0;
  for (int o : outs) bytes += f_.value_types[o].numel() * dtype_bytes(f_.value_types[o].dtype);
  for (int l : c.leaves) bytes += f_.value_types[l].numel() * dtype_bytes(f_.value_types[l].dtype);
  st->bytes_moved = bytes;
  return true;
}

std::string CodeGen::store(const Op& root, const std::string& expr) const {
  if (root.type.dtype == DType::BF16) return "sb_bf16_bits(" + expr + ")";
  if (root.type.dtype == DType::F32 &&
      std::find(round_roots_.begin(), round_roots_.end(), root.result) != round_roots_.end())
    return "sb_rna_tf32(" + expr + ")";
  return expr;
}

std::string CodeGen::source() const { return prelude() + src_.str(); }

}  // namespace sb
