// StableHLO text parser for the op forms Sheaf's emitter writes.
// Format references: sheaf/src/lowering/stablehlo/emit.rs:9-289 (module, func, return),
// operations.rs, broadcast.rs, reduce_ops.rs, shape_ops.rs, compare_ops.rs,
// tensor_ops.rs, dot_ops.rs, indexing_ops.rs, constants.rs; pad from
// sheaf/src/lowering/codegen/builtins.rs:228-296.
#include <cctype>
#include <cmath>
#include <cstring>
#include <sstream>
#include <stdexcept>
#include <unordered_map>

#include "ir.h"

namespace sb {

const char* dtype_name(DType t) {
  switch (t) {
    case DType::F32: return "f32";
    case DType::BF16: return "bf16";
    case DType::F64: return "f64";
    case DType::I32: return "i32";
    case DType::I64: return "i64";
    case DType::I1: return "i1";
  }
  return "?";
}

std::string Type::str() const {
  std::string s = "tensor<";
  for (auto d : shape) s += std::to_string(d) + "x";
  s += dtype_name(dtype);
  return s + ">";
}

const char* opkind_name(OpKind k) {
  static const char* names[] = {
      "constant", "add", "subtract", "multiply", "divide", "power", "maximum", "minimum",
      "remainder", "and", "or", "tanh", "sqrt", "rsqrt", "exponential", "log", "abs",
      "negate", "sine", "cosine", "not", "sign", "floor", "ceil", "logistic", "clamp",
      "convert", "select", "compare", "broadcast_in_dim", "reshape", "transpose", "iota",
      "slice", "pad", "concatenate", "reverse", "reduce", "dot_general", "gather",
      "attention_fwd", "attention_bwd", "bitcast_convert", "sort", "strided_view", "scatter_add_rows"};
  return names[(int)k];
}

const Function* Module::find(const std::string& q) const {
  for (auto& f : funcs) {
    if (f.name == q) return &f;
    if (!name.empty() && name + "." + f.name == q) return &f;
  }
  return nullptr;
}

namespace {

struct ParseError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

class Cursor {
 public:
  explicit Cursor(const std::string& s) : s_(s) {}

  void skip_ws() {
    for (;;) {
      while (i_ < s_.size() && std::isspace((unsigned char)s_[i_])) {
        if (s_[i_] == '\n') ++line_;
        ++i_;
      }
      if (i_ + 1 < s_.size() && s_[i_] == '/' && s_[i_ + 1] == '/') {
        while (i_ < s_.size() && s_[i_] != '\n') ++i_;
        continue;
      }
      break;
    }
  }
  bool eof() { skip_ws(); return i_ >= s_.size(); }
  bool peek(const char* t) {
    skip_ws();
    return s_.compare(i_, std::strlen(t), t) == 0;
  }
  bool accept(const char* t) {
    if (peek(t)) { i_ += std::strlen(t); return true; }
    return false;
  }
  void expect(const char* t) {
    if (!accept(t)) fail(std::string("expected '") + t + "'");
  }
  [[noreturn]] void fail(const std::string& msg) {
    size_t e = s_.find('\n', i_);
    std::string ctx = s_.substr(i_, std::min<size_t>(e == std::string::npos ? 60 : e - i_, 60));
    throw ParseError("line " + std::to_string(line_) + ": " + msg + " near '" + ctx + "'");
  }
  int line() const { return line_; }

  std::string ident() {  // [A-Za-z_][A-Za-z0-9_.$-]*
    skip_ws();
    size_t b = i_;
    while (i_ < s_.size() && (std::isalnum((unsigned char)s_[i_]) || s_[i_] == '_' ||
                              s_[i_] == '.' || s_[i_] == '$' || s_[i_] == '-'))
      ++i_;
    if (b == i_) fail("expected identifier");
    return s_.substr(b, i_ - b);
  }
  std::string value_name() {  // %name
    skip_ws();
    if (i_ >= s_.size() || s_[i_] != '%') fail("expected %value");
    size_t b = i_++;
    while (i_ < s_.size() && (std::isalnum((unsigned char)s_[i_]) || s_[i_] == '_')) ++i_;
    return s_.substr(b, i_ - b);
  }
  int64_t integer() {
    skip_ws();
    size_t b = i_;
    if (i_ < s_.size() && (s_[i_] == '-' || s_[i_] == '+')) ++i_;
    while (i_ < s_.size() && std::isdigit((unsigned char)s_[i_])) ++i_;
    if (b == i_) fail("expected integer");
    return std::stoll(s_.substr(b, i_ - b));
  }
  double number() {
    skip_ws();
    size_t b = i_;
    if (s_.compare(i_, 2, "0x") == 0 || s_.compare(i_, 2, "0X") == 0) {
      i_ += 2;
      while (i_ < s_.size() && std::isxdigit((unsigned char)s_[i_])) ++i_;
      uint64_t bits = std::stoull(s_.substr(b + 2, i_ - b - 2), nullptr, 16);
      if (i_ - b - 2 <= 8) {
        uint32_t u = (uint32_t)bits;
        float f;
        std::memcpy(&f, &u, 4);
        return f;
      }
      double d;
      std::memcpy(&d, &bits, 8);
      return d;
    }
    if (s_.compare(i_, 4, "true") == 0) { i_ += 4; return 1.0; }
    if (s_.compare(i_, 5, "false") == 0) { i_ += 5; return 0.0; }
    while (i_ < s_.size() && (std::isdigit((unsigned char)s_[i_]) || s_[i_] == '.' || s_[i_] == '-' ||
                              s_[i_] == '+' || s_[i_] == 'e' || s_[i_] == 'E' || s_[i_] == 'n' ||
                              s_[i_] == 'a' || s_[i_] == 'i' || s_[i_] == 'f'))
      ++i_;
    if (b == i_) fail("expected number");
    std::string t = s_.substr(b, i_ - b);
    try {
      return std::stod(t);
    } catch (...) {
      fail("bad number '" + t + "'");
    }
  }
  std::vector<int64_t> int_list() {  // [a, b, c]
    expect("[");
    std::vector<int64_t> v;
    if (accept("]")) return v;
    do { v.push_back(integer()); } while (accept(","));
    expect("]");
    return v;
  }
  Type type() {
    expect("tensor<");
    size_t e = s_.find('>', i_);
    if (e == std::string::npos) fail("unterminated tensor type");
    std::string inner = s_.substr(i_, e - i_);
    i_ = e + 1;
    Type t;
    std::vector<std::string> parts;
    size_t p = 0;
    for (;;) {
      size_t q = inner.find('x', p);
      // the element type may itself contain no 'x'; dims are digits
      if (q == std::string::npos || !std::isdigit((unsigned char)inner[p])) {
        parts.push_back(inner.substr(p));
        break;
      }
      parts.push_back(inner.substr(p, q - p));
      p = q + 1;
    }
    for (size_t k = 0; k + 1 < parts.size(); ++k) t.shape.push_back(std::stoll(parts[k]));
    const std::string& et = parts.back();
    if (et == "f32") t.dtype = DType::F32;
    else if (et == "bf16") t.dtype = DType::BF16;
    else if (et == "f64") t.dtype = DType::F64;
    else if (et == "i32" || et == "ui32") t.dtype = DType::I32;
    else if (et == "i64" || et == "ui64") t.dtype = DType::I64;
    else if (et == "i1") t.dtype = DType::I1;
    else fail("unsupported element type '" + et + "'");
    return t;
  }
  // Raw text up to (not including) the matching close of an open bracket already consumed.
  void skip_balanced(char open, char close) {
    int depth = 1;
    while (i_ < s_.size() && depth) {
      if (s_[i_] == '\n') ++line_;
      if (s_[i_] == open) ++depth;
      else if (s_[i_] == close) --depth;
      ++i_;
    }
  }
  size_t pos() const { return i_; }
  void set_pos(size_t p) { i_ = p; }
  const std::string& src() const { return s_; }

 private:
  const std::string& s_;
  size_t i_ = 0;
  int line_ = 1;
};

struct FuncBuilder {
  Function f;
  std::unordered_map<std::string, int> ids;
  Cursor& c;
  explicit FuncBuilder(Cursor& cur) : c(cur) {}

  int define(const std::string& name, const Type& t) {
    if (ids.count(name)) c.fail("redefinition of " + name);
    int id = (int)f.value_types.size();
    ids[name] = id;
    f.value_types.push_back(t);
    return id;
  }
  int use(const std::string& name) {
    auto it = ids.find(name);
    if (it == ids.end()) c.fail("use of undefined value " + name);
    return it->second;
  }
  int use_next() { return use(c.value_name()); }
};

void parse_dense(Cursor& c, Op& op) {
  // dense<v> | dense<[..nested..]> | dense<0xFF800000>
  c.expect("dense<");
  if (c.peek("[")) {
    int depth = 0;
    do {
      if (c.accept("[")) { ++depth; continue; }
      if (c.accept("]")) { --depth; continue; }
      if (c.accept(",")) continue;
      op.values.push_back(c.number());
    } while (depth > 0);
  } else {
    op.values.push_back(c.number());
  }
  c.expect(">");
}

OpKind elementwise_kind(const std::string& n, bool* ok) {
  static const std::unordered_map<std::string, OpKind> m = {
      {"add", OpKind::Add}, {"subtract", OpKind::Sub}, {"multiply", OpKind::Mul},
      {"divide", OpKind::Div}, {"power", OpKind::Pow}, {"maximum", OpKind::Max},
      {"minimum", OpKind::Min}, {"remainder", OpKind::Rem}, {"and", OpKind::And},
      {"or", OpKind::Or}, {"tanh", OpKind::Tanh}, {"sqrt", OpKind::Sqrt},
      {"rsqrt", OpKind::Rsqrt}, {"exponential", OpKind::Exp}, {"log", OpKind::Log},
      {"abs", OpKind::Abs}, {"negate", OpKind::Neg}, {"sine", OpKind::Sin},
      {"cosine", OpKind::Cos}, {"not", OpKind::Not}, {"sign", OpKind::Sign},
      {"floor", OpKind::Floor}, {"ceil", OpKind::Ceil}, {"logistic", OpKind::Logistic}};
  auto it = m.find(n);
  *ok = it != m.end();
  return *ok ? it->second : OpKind::Add;
}

// %v, %i = "stablehlo.sort"(%keys, %payload) ({ ^bb0(...): compare GT|LT of
// the first two block arguments; return }) {dimension = last, is_stable} as
// emitted for top_k (lowering/stablehlo/indexing_ops.rs:476-540).
void parse_sort(FuncBuilder& fb, Cursor& c, const std::vector<std::string>& results, int line) {
  c.expect("\"stablehlo.sort\"");
  c.expect("(");
  const int x = fb.use_next();
  c.expect(",");
  const int pay = fb.use_next();
  c.expect(")");
  c.expect("(");
  c.expect("{");
  c.expect("^bb0(");
  std::vector<std::string> args;
  do {
    args.push_back(c.value_name());
    c.expect(":");
    c.type();
  } while (c.accept(","));
  c.expect(")");
  c.expect(":");
  const std::string p = c.value_name();
  c.expect("=");
  c.expect("\"stablehlo.compare\"");
  c.expect("(");
  const std::string l = c.value_name();
  c.expect(",");
  const std::string r = c.value_name();
  c.expect(")");
  c.expect("{");
  c.expect("comparison_direction");
  c.expect("=");
  c.expect("#stablehlo<comparison_direction");
  const std::string dir = c.ident();
  c.expect(">");
  if (c.accept(",")) {  // compare_type = #stablehlo<comparison_type FLOAT>
    c.ident();
    c.expect("=");
    c.expect("#stablehlo<comparison_type");
    c.ident();
    c.expect(">");
  }
  c.expect("}");
  c.expect(":");
  c.expect("(");
  c.type();
  c.expect(",");
  c.type();
  c.expect(")");
  c.expect("->");
  c.type();
  c.expect("\"stablehlo.return\"");
  c.expect("(");
  const std::string rv = c.value_name();
  c.expect(")");
  c.expect(":");
  c.expect("(");
  c.type();
  c.expect(")");
  c.expect("->");
  c.expect("(");
  c.expect(")");
  c.expect("}");
  c.expect(")");
  c.expect("{");
  c.expect("dimension");
  c.expect("=");
  const int64_t dim = c.integer();
  c.expect(":");
  c.ident();
  if (c.accept(",")) {
    c.expect("is_stable");
    c.expect("=");
    c.ident();  // the kernel is stable either way
  }
  c.expect("}");
  c.expect(":");
  c.expect("(");
  const Type tx = c.type();
  c.expect(",");
  const Type tp = c.type();
  c.expect(")");
  c.expect("->");
  c.expect("(");
  const Type ta = c.type();
  c.expect(",");
  const Type tb = c.type();
  c.expect(")");
  if (args.size() != 4 || l != args[0] || r != args[1] || rv != p || (dir != "GT" && dir != "LT"))
    c.fail("sort: only a GT / LT comparator on the first operand is supported");
  if (tx.dtype != DType::F32 || tp.dtype != DType::I32 || ta.shape != tx.shape || tb.shape != tp.shape ||
      tp.shape != tx.shape || ta.dtype != DType::F32 || tb.dtype != DType::I32)
    c.fail("sort: operands must be (f32 keys, i32 payload) of one shape");
  if (tx.shape.empty() || dim != (int64_t)tx.shape.size() - 1) c.fail("sort: only the last dimension is supported");
  const int64_t n = tx.shape.back();
  Op s;
  s.kind = OpKind::SortPairs;
  s.line = line;
  s.operands = {x, pay};
  s.axis = dir == "GT" ? 1 : 0;
  s.type = tx;
  s.type.shape.back() = 2 * n;
  s.result = fb.define(results[0] + "$packed", s.type);
  const int packed = s.result;
  fb.f.ops.push_back(s);
  auto half = [&](int64_t lo, const std::string& name) {
    Op h;
    h.kind = OpKind::Slice;
    h.line = line;
    h.operands = {packed};
    for (size_t d = 0; d < tx.shape.size(); ++d) {
      const bool last = d + 1 == tx.shape.size();
      h.a0.push_back(last ? lo : 0);
      h.a1.push_back(last ? lo + n : tx.shape[d]);
      h.a2.push_back(1);
    }
    h.type = tx;
    h.result = fb.define(name, tx);
    fb.f.ops.push_back(h);
    return h.result;
  };
  half(0, results[0]);
  const int bits = half(n, results[1] + "$bits");
  Op b;
  b.kind = OpKind::Bitcast;
  b.line = line;
  b.operands = {bits};
  b.type = tp;
  b.result = fb.define(results[1], tp);
  fb.f.ops.push_back(b);
}

void parse_statement(FuncBuilder& fb, Cursor& c) {
  int line = c.line();
  std::vector<std::string> results;
  results.push_back(c.value_name());
  while (c.accept(",")) results.push_back(c.value_name());
  c.expect("=");
  if (results.size() == 2 && c.peek("\"stablehlo.sort\"")) {
    parse_sort(fb, c, results, line);
    return;
  }
  Op op;
  op.line = line;
  if (results.size() != 1) c.fail("multi-result ops are not supported");

  if (c.accept("\"stablehlo.gather\"")) {
    op.kind = OpKind::Gather;
    c.expect("(");
    op.operands.push_back(fb.use_next());
    c.expect(",");
    op.operands.push_back(fb.use_next());
    c.expect(")");
    c.expect("{");
    // attributes
    c.expect("dimension_numbers");
    c.expect("=");
    c.expect("#stablehlo.gather<");
    while (!c.accept(">")) {
      std::string key = c.ident();
      c.expect("=");
      if (key == "index_vector_dim") op.axis = c.integer();
      else {
        auto v = c.int_list();
        if (key == "offset_dims") op.offset_dims = v;
        else if (key == "collapsed_slice_dims") op.collapsed = v;
        else if (key == "start_index_map") op.start_index_map = v;
        else if (key == "operand_batching_dims" || key == "start_indices_batching_dims") {
          if (!v.empty()) c.fail("gather batching dims are not supported");
        } else c.fail("unknown gather attribute " + key);
      }
      c.accept(",");
    }
    c.accept(",");
    while (!c.accept("}")) {
      std::string key = c.ident();
      c.expect("=");
      if (key == "slice_sizes") {
        c.expect("array<i64:");
        do { op.slice_sizes.push_back(c.integer()); } while (c.accept(","));
        c.expect(">");
      } else if (key == "indices_are_sorted") {
        c.ident();
      } else c.fail("unknown gather attribute " + key);
      c.accept(",");
    }
    c.expect(":");
    c.expect("(");
    c.type();
    c.expect(",");
    c.type();
    c.expect(")");
    c.expect("->");
    op.type = c.type();
  } else {
    std::string name = c.ident();
    if (name.rfind("stablehlo.", 0) != 0) c.fail("unsupported operation '" + name + "'");
    std::string k = name.substr(10);
    bool ew = false;
    OpKind ek = elementwise_kind(k, &ew);
    if (k == "constant") {
      op.kind = OpKind::Constant;
      parse_dense(c, op);
      c.expect(":");
      op.type = c.type();
      if (op.values.size() != 1 && (int64_t)op.values.size() != op.type.numel())
        c.fail("constant payload size does not match its type");
    } else if (ew) {
      op.kind = ek;
      op.operands.push_back(fb.use_next());
      if (is_binary_elementwise(ek)) {
        c.expect(",");
        op.operands.push_back(fb.use_next());
      }
      c.expect(":");
      op.type = c.type();
    } else if (k == "clamp") {
      op.kind = OpKind::Clamp;
      for (int j = 0; j < 3; ++j) {
        if (j) c.expect(",");
        op.operands.push_back(fb.use_next());
      }
      c.expect(":");
      op.type = c.type();
    } else if (k == "convert" || k == "reshape" || k == "bitcast_convert") {
      op.kind = k == "convert" ? OpKind::Convert : k == "reshape" ? OpKind::Reshape : OpKind::Bitcast;
      op.operands.push_back(fb.use_next());
      c.expect(":");
      c.expect("(");
      c.type();
      c.expect(")");
      c.expect("->");
      op.type = c.type();
    } else if (k == "broadcast_in_dim" || k == "transpose" || k == "reverse") {
      op.kind = k == "broadcast_in_dim" ? OpKind::BroadcastInDim
                : k == "transpose" ? OpKind::Transpose : OpKind::Reverse;
      op.operands.push_back(fb.use_next());
      c.expect(",");
      c.expect("dims");
      c.expect("=");
      op.dims = c.int_list();
      c.expect(":");
      c.expect("(");
      c.type();
      c.expect(")");
      c.expect("->");
      op.type = c.type();
    } else if (k == "reduce") {
      op.kind = OpKind::Reduce;
      c.expect("(");
      op.operands.push_back(fb.use_next());
      c.expect("init:");
      op.operands.push_back(fb.use_next());
      c.expect(")");
      c.expect("applies");
      std::string b = c.ident();
      if (b == "stablehlo.add") op.body = ReduceBody::Add;
      else if (b == "stablehlo.maximum") op.body = ReduceBody::Max;
      else if (b == "stablehlo.minimum") op.body = ReduceBody::Min;
      else if (b == "stablehlo.multiply") op.body = ReduceBody::Mul;
      else c.fail("unsupported reduce body " + b);
      c.expect("across");
      c.expect("dimensions");
      c.expect("=");
      op.dims = c.int_list();
      c.expect(":");
      c.expect("(");
      c.type();
      c.expect(",");
      c.type();
      c.expect(")");
      c.expect("->");
      op.type = c.type();
    } else if (k == "iota") {
      op.kind = OpKind::Iota;
      c.expect("dim");
      c.expect("=");
      op.axis = c.integer();
      c.expect(":");
      op.type = c.type();
    } else if (k == "dot_general") {
      op.kind = OpKind::DotGeneral;
      op.operands.push_back(fb.use_next());
      c.expect(",");
      op.operands.push_back(fb.use_next());
      c.expect(",");
      if (c.accept("batching_dims")) {
        c.expect("=");
        op.lb = c.int_list();
        c.expect("x");
        op.rb = c.int_list();
        c.expect(",");
      }
      c.expect("contracting_dims");
      c.expect("=");
      op.lc = c.int_list();
      c.expect("x");
      op.rc = c.int_list();
      if (c.accept(",")) {  // optional precision = [...] etc.: skip to ':'
        while (!c.peek(":")) c.ident();
      }
      c.expect(":");
      c.expect("(");
      c.type();
      c.expect(",");
      c.type();
      c.expect(")");
      c.expect("->");
      op.type = c.type();
    } else if (k == "compare") {
      op.kind = OpKind::Compare;
      std::string d = c.ident();
      if (d == "EQ") op.cmp = CmpDir::EQ;
      else if (d == "NE") op.cmp = CmpDir::NE;
      else if (d == "LT") op.cmp = CmpDir::LT;
      else if (d == "LE") op.cmp = CmpDir::LE;
      else if (d == "GT") op.cmp = CmpDir::GT;
      else if (d == "GE") op.cmp = CmpDir::GE;
      else c.fail("bad comparison direction " + d);
      c.expect(",");
      op.operands.push_back(fb.use_next());
      c.expect(",");
      op.operands.push_back(fb.use_next());
      if (c.accept(",")) c.ident();  // FLOAT / SIGNED / ...
      c.expect(":");
      c.expect("(");
      c.type();
      c.expect(",");
      c.type();
      c.expect(")");
      c.expect("->");
      op.type = c.type();
    } else if (k == "select") {
      op.kind = OpKind::Select;
      for (int j = 0; j < 3; ++j) {
        if (j) c.expect(",");
        op.operands.push_back(fb.use_next());
      }
      c.expect(":");
      Type t0 = c.type();
      if (c.accept(",")) op.type = c.type();
      else op.type = t0;
    } else if (k == "slice") {
      op.kind = OpKind::Slice;
      op.operands.push_back(fb.use_next());
      c.expect("[");
      if (!c.accept("]")) {
        do {
          op.a0.push_back(c.integer());
          c.expect(":");
          op.a1.push_back(c.integer());
          if (c.accept(":")) op.a2.push_back(c.integer());
          else op.a2.push_back(1);
        } while (c.accept(","));
        c.expect("]");
      }
      c.expect(":");
      c.expect("(");
      c.type();
      c.expect(")");
      c.expect("->");
      op.type = c.type();
    } else if (k == "pad") {
      op.kind = OpKind::Pad;
      op.operands.push_back(fb.use_next());
      c.expect(",");
      op.operands.push_back(fb.use_next());
      c.expect(",");
      c.expect("low");
      c.expect("=");
      op.a0 = c.int_list();
      c.expect(",");
      c.expect("high");
      c.expect("=");
      op.a1 = c.int_list();
      c.expect(",");
      c.expect("interior");
      c.expect("=");
      op.a2 = c.int_list();
      c.expect(":");
      c.expect("(");
      c.type();
      c.expect(",");
      c.type();
      c.expect(")");
      c.expect("->");
      op.type = c.type();
    } else if (k == "concatenate") {
      op.kind = OpKind::Concatenate;
      op.operands.push_back(fb.use_next());
      while (c.accept(",")) {
        if (c.accept("dim")) break;
        op.operands.push_back(fb.use_next());
      }
      c.expect("=");
      op.axis = c.integer();
      c.expect(":");
      c.expect("(");
      c.skip_balanced('(', ')');
      c.expect("->");
      op.type = c.type();
    } else {
      c.fail("unsupported operation '" + name + "'");
    }
  }
  op.result = fb.define(results[0], op.type);
  fb.f.ops.push_back(std::move(op));
}

void parse_function(Module& m, Cursor& c) {
  FuncBuilder fb(c);
  c.expect("func.func");
  if (c.accept("private")) {}
  c.expect("@");
  fb.f.name = c.ident();
  c.expect("(");
  if (!c.accept(")")) {
    do {
      std::string n = c.value_name();
      c.expect(":");
      Type t = c.type();
      fb.f.params.push_back(t);
      fb.define(n, t);
    } while (c.accept(","));
    c.expect(")");
  }
  c.expect("->");
  if (c.accept("(")) {
    if (!c.accept(")")) {
      do { fb.f.results.push_back(c.type()); } while (c.accept(","));
      c.expect(")");
    }
  } else {
    fb.f.results.push_back(c.type());
  }
  c.expect("{");
  for (;;) {
    if (c.accept("}")) break;
    if (c.accept("return")) {
      if (!c.peek(":") && !c.peek("}")) {
        do { fb.f.returns.push_back(fb.use_next()); } while (c.accept(","));
      }
      if (c.accept(":")) {
        for (size_t j = 0; j < fb.f.returns.size(); ++j) {
          if (j) c.expect(",");
          c.type();
        }
      }
      continue;
    }
    if (c.peek("%")) {
      parse_statement(fb, c);
      continue;
    }
    c.fail("unexpected token in function body");
  }
  if (fb.f.returns.size() != fb.f.results.size())
    c.fail("return arity does not match the function signature of @" + fb.f.name);
  for (size_t j = 0; j < fb.f.returns.size(); ++j)
    if (!(fb.f.value_types[fb.f.returns[j]].shape == fb.f.results[j].shape))
      c.fail("return type mismatch in @" + fb.f.name);
  fb.f.producer.assign(fb.f.value_types.size(), -1);
  for (size_t j = 0; j < fb.f.ops.size(); ++j) fb.f.producer[fb.f.ops[j].result] = (int)j;
  m.funcs.push_back(std::move(fb.f));
}

}  // namespace

std::unique_ptr<Module> parse_module(const std::string& text, std::string* error) {
  auto m = std::make_unique<Module>();
  Cursor c(text);
  try {
    c.expect("module");
    if (c.accept("@")) m->name = c.ident();
    c.expect("{");
    while (!c.accept("}")) {
      if (c.peek("func.func")) parse_function(*m, c);
      else c.fail("expected func.func");
    }
    if (!c.eof()) c.fail("trailing text after module");
    if (m->funcs.empty()) c.fail("module has no functions");
  } catch (const ParseError& e) {
    if (error) *error = std::string("StableHLO parse error: ") + e.what();
    return nullptr;
  }
  return m;
}

}  // namespace sb
