// CUDA C++ generation for fused clusters (loop fusion and reduction input fusion).
// Shapes are static, so every extent and stride is baked into the kernel text.
#pragma once
#include <map>
#include <sstream>
#include <string>
#include <vector>

#include "ir.h"
#include "plan.h"

namespace sb {

class CodeGen {
 public:
  // cluster[v]: root value id for fused/root nodes, negative for duplicable (-2),
  // dense constant (-3) and parameter (-4) values.
  CodeGen(const Function& f, const std::vector<int>& cluster) : f_(f), cluster_(cluster) {}
  // Roots whose stored values are rounded to nearest TF32 (they feed tf32 GEMMs;
  // the tensor cores would otherwise truncate them).
  void set_round_roots(const std::vector<int>& roots) { round_roots_ = roots; }
  // Values whose GEMM operand shadow (a TF32-rounded f32 or a bf16 copy) the
  // producing row-group kernel writes as well, as it stores the value
  // (Step::shadow_values); others get a separate conversion step.
  void set_shadow_values(const std::map<int, DType>& v) { shadow_vals_ = v; }

  void gen_loop(const Op& root, Step* st);
  // Reduction `root`; with `epi`, the element-wise cluster rooted at epi (of
  // root's shape, reading root at the output coordinates) is evaluated on each
  // reduced value and stored instead.
  void gen_reduce(const Op& root, Step* st, const Op* epi = nullptr);
  // A row group: steps over the same R rows of C columns, run back to back
  // for each row by one warp in a single kernel.  kind 0: loop over
  // [rows..., C]; 1: loop over the rows (R elements); 2: reduction over the
  // innermost C of a [rows..., C] operand (root = the reduce op, optional
  // element-wise epilogue epi).  Later members read earlier members' outputs
  // only at their own row (the caller checks), after a __syncwarp.  Returns
  // false (nothing emitted) when a member does not fit the scheme.
  struct RowMember {
    int kind;
    const Op* root;
    const Op* epi;
  };
  bool gen_row_group(const std::vector<RowMember>& ms, int64_t R, int64_t C, Step* st);
  std::string source() const;
  static std::string prelude();
  std::vector<std::string> kernel_names() const { return names_; }
  const std::vector<std::string>& snippets() const { return snippets_; }

 private:
  struct Val {
    std::string name;
    std::string ctype;
  };
  struct Ctx {
    int root = -1;
    std::vector<int> leaves;
    std::map<int, int> leaf_index;
    std::ostringstream body;
    int tmp = 0;
    int indent = 2;
    std::string idx;  // index C type
    std::vector<std::map<std::string, Val>> memo;
    // 4-wide mode: the innermost output coordinate of lane j is "cL" (j = 0)
    // or "(cL+j)"; contiguous f32 leaf reads become one float4 load per lane group
    bool vec = false;
    std::map<std::string, std::string> vloads;  // leaf:offset -> float4 variable
    // row groups: outputs of earlier members held in registers (value ->
    // 0: one register per row element of this lane, 1: one per row) and the
    // registers, keyed "<value>@<lane base>:<k>" or "<value>@row"
    std::map<int, int> reg_kind;
    std::map<std::string, Val> regs;
    std::string pad() const { return std::string(indent * 2, ' '); }
  };

  bool gen_loop_vec4(const Op& root, Step* st);
  bool gen_reduce_vec4(const Op& root, Step* st, const Op* epi);
  // Code of the epilogue expression at output coordinates oc, with the
  // reduced value in the variable r_; *val receives its name.
  std::string epilogue_code(Ctx& c, const Op& red, const Op& epi, const std::vector<std::string>& oc, int indent,
                            std::string* val, const std::string& rv = "rv_");
  Val eval(Ctx& c, int v, const std::vector<std::string>& coords);
  Val leaf_load(Ctx& c, int v, const std::vector<std::string>& coords);
  std::string fresh(Ctx& c, const char* p = "t") { return p + std::to_string(c.tmp++); }
  bool is_materialized_for(const Ctx& c, int v) const;
  std::string header(const std::string& name, const Ctx& c, int extra_ptrs) const;
  std::string index_type(const Op& root, int64_t extra) const;

  const Function& f_;
  const std::vector<int>& cluster_;
  std::ostringstream src_;
  std::string store(const Op& root, const std::string& expr) const;

  std::vector<std::string> names_;
  std::vector<std::string> snippets_;
  std::vector<int> round_roots_;
  std::map<int, DType> shadow_vals_;
};

const char* ctype_of(DType t);

}  // namespace sb
