// In-memory form of a parsed StableHLO module (the subset Sheaf's emitter writes,
// sheaf/src/lowering/stablehlo/*.rs).  One Function per `func.func`; SSA values
// are dense integer ids, parameters first.
#pragma once
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace sb {

enum class DType : uint8_t { F32, BF16, F64, I32, I64, I1 };

inline int dtype_bytes(DType t) {
  switch (t) {
    case DType::F32: case DType::I32: return 4;
    case DType::BF16: return 2;
    case DType::F64: case DType::I64: return 8;
    case DType::I1: return 1;
  }
  return 4;
}
inline bool dtype_is_float(DType t) { return t == DType::F32 || t == DType::BF16 || t == DType::F64; }
const char* dtype_name(DType t);

struct Type {
  std::vector<int64_t> shape;
  DType dtype = DType::F32;
  int64_t numel() const {
    int64_t n = 1;
    for (auto d : shape) n *= d;
    return n;
  }
  int rank() const { return (int)shape.size(); }
  bool operator==(const Type& o) const { return shape == o.shape && dtype == o.dtype; }
  std::string str() const;
};

enum class OpKind : uint8_t {
  Constant, Add, Sub, Mul, Div, Pow, Max, Min, Rem, And, Or,
  Tanh, Sqrt, Rsqrt, Exp, Log, Abs, Neg, Sin, Cos, Not, Sign, Floor, Ceil, Logistic,
  Clamp, Convert, Select, Compare,
  BroadcastInDim, Reshape, Transpose, Iota, Slice, Pad, Concatenate, Reverse,
  Reduce, DotGeneral, Gather,
  // Fused attention (head dim 64), created by the planner's attention rewrite,
  // never parsed.  Operands: q, k, v [B,H,T,64] (+ dy, y [B,H,T,64] and
  // lse [B,H,T] for AttnBwd).  values[0] = score scale, axis = causal.
  // Results are packed 1-D buffers: AttnFwd [Y (B,T,H,64) | L (B,H,T)],
  // AttnBwd [dQ, dK, dV interleaved as (B,T,3,H,64) | D (B,H,T)].
  AttnFwd, AttnBwd,
  // stablehlo.bitcast_convert between 32-bit element types (f32 <-> i32)
  Bitcast,
  // stablehlo.sort of (f32 keys, i32 payload) along the last dim with a
  // GT / LT comparator on the keys, stable.  Created by the parser: the op
  // writes one packed f32 buffer [.., 2N] (sorted keys | payload bits) and
  // the two results are a slice and a bitcast slice of it.  axis = 1 for
  // descending (GT).
  SortPairs,
  // As-strided view of the row-major flattening of its operand, created by
  // the planner's sibling-GEMM merge, never parsed: element i of the result
  // is operand_flat[a0[0] + sum_d i_d * a2[d]].  A pure index map.
  StridedView,
  // Row scatter-add, created by the planner's embedding-gradient rewrite,
  // never parsed.  Operands: idx (n index values, f32 or i32), adj (n rows of
  // d, row-major).  Result [V, d]: row k = sum of the adj rows whose index is
  // k, in row order (indices that are not integers in [0, V) hit no row).
  ScatterAddRows,
};
const char* opkind_name(OpKind k);

inline bool is_binary_elementwise(OpKind k) {
  return k == OpKind::Add || k == OpKind::Sub || k == OpKind::Mul || k == OpKind::Div ||
         k == OpKind::Pow || k == OpKind::Max || k == OpKind::Min || k == OpKind::Rem ||
         k == OpKind::And || k == OpKind::Or;
}
inline bool is_unary_elementwise(OpKind k) {
  return k == OpKind::Tanh || k == OpKind::Sqrt || k == OpKind::Rsqrt || k == OpKind::Exp ||
         k == OpKind::Log || k == OpKind::Abs || k == OpKind::Neg || k == OpKind::Sin ||
         k == OpKind::Cos || k == OpKind::Not || k == OpKind::Sign || k == OpKind::Floor ||
         k == OpKind::Ceil || k == OpKind::Logistic || k == OpKind::Convert || k == OpKind::Bitcast;
}
inline bool is_attention(OpKind k) {
  return k == OpKind::AttnFwd || k == OpKind::AttnBwd;
}
inline bool is_elementwise(OpKind k) {
  return is_binary_elementwise(k) || is_unary_elementwise(k) || k == OpKind::Clamp ||
         k == OpKind::Select || k == OpKind::Compare;
}

enum class CmpDir : uint8_t { EQ, NE, LT, LE, GT, GE };
enum class ReduceBody : uint8_t { Add, Max, Min, Mul };

struct Op {
  OpKind kind;
  int result = -1;               // value id
  std::vector<int> operands;     // value ids
  Type type;                     // result type
  int line = 0;                  // source line, for diagnostics
  // attributes (meaning depends on kind)
  std::vector<int64_t> dims;     // broadcast dims / transpose perm / reduce dims / reverse dims
  std::vector<int64_t> a0, a1, a2;  // slice start/limit/stride; pad low/high/interior
  std::vector<int64_t> lb, rb, lc, rc;  // dot_general batching/contracting dims
  int64_t axis = 0;              // iota dim / concatenate dim / gather index_vector_dim
  CmpDir cmp = CmpDir::EQ;
  ReduceBody body = ReduceBody::Add;
  std::vector<double> values;    // constant payload (size 1 = splat)
  std::vector<int64_t> offset_dims, collapsed, start_index_map, slice_sizes;  // gather
};

struct Function {
  std::string name;
  std::vector<Type> params;
  std::vector<Type> results;
  std::vector<Op> ops;
  std::vector<int> returns;      // value ids
  std::vector<Type> value_types; // indexed by value id
  std::vector<int> producer;     // value id -> op index (-1 for params)
  int num_values() const { return (int)value_types.size(); }
};

struct Module {
  std::string name;
  std::vector<Function> funcs;
  const Function* find(const std::string& qualified) const;
};

// Parses StableHLO text.  On failure returns nullptr and sets *error.
std::unique_ptr<Module> parse_module(const std::string& text, std::string* error);

}  // namespace sb
