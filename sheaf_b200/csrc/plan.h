// Execution plan for one StableHLO function: fusion clusters, GEMM steps,
// memory layout of intermediates, and the CUDA source of the fused kernels.
#pragma once
#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "ir.h"

namespace sb {

enum class Precision : int { FP32 = 0, TF32 = 1, BF16 = 2 };

// Affine view of a materialized buffer: element (i0..in) lives at
// base[offset + sum(i_k * strides[k])].
struct View {
  int value = -1;  // materialized value id (param, constant or step root)
  int64_t offset = 0;
  std::vector<int64_t> shape, strides;
};

// Batched GEMM C[b,m,n] = sum_k A[b,m,k] * B[b,k,n]; strides in elements.
struct GemmDesc {
  View a, b;
  int64_t batch = 1, M = 1, N = 1, K = 1;
  int64_t sab = 0, sam = 0, sak = 0;
  int64_t sbb = 0, sbk = 0, sbn = 0;
  bool a_rounded = false, b_rounded = false;  // read the TF32-rounded copy of a parameter
  bool round_out = false;                     // store the result rounded to TF32
  int a_shadow = -1, b_shadow = -1;           // read operand shadow Plan::shadows[i] instead
  bool bf16 = false;                          // both operands are read as bf16
  // fused epilogue (kEpiGelu): the step also writes Step::extra_roots[0] =
  // gelu(result), rounded to TF32 when round_out2
  int epi = 0;
  bool round_out2 = false;
};

// Copy of a GEMM operand in the form the tensor cores read, written by a
// conversion step right after the step that produces the value (parameters:
// first in the call): f32 rounded to nearest TF32 (TF32 mode, for operands
// that other steps also read, so that their producer cannot store them
// rounded), or bf16 (bf16 mode, every f32 GEMM operand).
struct Shadow {
  int value = -1;       // the materialized value copied
  int step = -1;        // the conversion step
  int last_use = -1;    // last step that reads the shadow
  int64_t offset = -1;  // arena byte offset
  DType dtype = DType::F32;
};

struct GatherDesc {
  int table = -1;
};

// Fused attention step (OpKind::AttnFwd / AttnBwd).  Operand
// views in the op's operand order; dims B, H, T, head dim 64.
struct AttnDesc {
  OpKind kind = OpKind::AttnFwd;
  std::vector<View> in;
  std::vector<char> rounded;  // per operand: read the TF32-rounded copy of a parameter
  int64_t B = 0, H = 0, T = 0;
  double scale = 1;
  bool causal = false;
  bool round_out = false;  // Y / dQ / dK / dV stored rounded to TF32
};

enum class StepKind : uint8_t { Loop, Reduce, Gemm, Attn, Sort, Convert, Scatter };

struct Step {
  StepKind kind = StepKind::Loop;
  int root = -1;                // value written by this step
  std::vector<int> extra_roots; // further values written (row groups), kernel arguments after root
  std::vector<int> leaves;      // materialized values read (kernel argument order)
  std::string kernel;           // generated kernel name (Loop / Reduce)
  int64_t grid = 1, block = 256, grid_y = 1;
  // split reduction: partial results go to scratch, a second kernel finishes
  std::string finish_kernel;
  int64_t finish_grid = 1, splits = 1, scratch_elems = 0;
  GemmDesc gemm;
  AttnDesc attn;
  int64_t elements = 0;         // output elements
  int64_t bytes_moved = 0;      // algorithmic bytes (inputs read once + output)
  double flops = 0;
  int shadow = -1;              // Convert: index into Plan::shadows
  // values whose operand shadows this step's kernel writes too (kernel
  // arguments after the root, the extra roots and the scratch), and those
  // shadows' indices into Plan::shadows, in the same order
  std::vector<int> shadow_values;
  std::vector<int> shadow_outs;
  // Column reductions of a row group whose finish is a plain column sum (f32,
  // zero init, no rounding): per reduction, its output's index among root and
  // extra roots and the offset (floats) of its block partials in the scratch.
  // With finish_deferred (no later step reads the outputs) the runtime may
  // add the partials later, batched with other steps' (col_sum_segments).
  struct ColFinish {
    int out = 0;
    int64_t offset = 0;
  };
  std::vector<ColFinish> col_finish;
  int64_t col_C = 0;
  bool finish_deferred = false;
};

struct Plan {
  const Function* fn = nullptr;       // the planned function (may be `rewritten`)
  std::shared_ptr<Function> rewritten;  // set when the attention rewrite applied
  std::string rewrite_log;
  std::vector<Step> steps;
  std::vector<int> materialized;      // values written by steps, in step order
  std::vector<int> constants;         // dense (non-splat) constants uploaded at load
  std::vector<int64_t> value_offset;  // arena byte offset per value (-1 if not in arena)
  std::vector<int64_t> scratch_offset;  // per step, arena offset of split-reduce scratch
  std::vector<int> output_step;       // per return slot: step that writes it (-1: copy)
  std::vector<int> rounded_params;    // parameters read by tf32 GEMMs through a rounded copy
  std::vector<int64_t> rounded_offset;  // arena offset of each rounded copy
  std::vector<Shadow> shadows;        // GEMM operand copies (see Shadow)
  int64_t arena_bytes = 0;
  std::string source;                 // CUDA C++ of all generated kernels
  std::vector<std::string> snippets;  // the same, one independent piece per step
  std::string prelude;                // helpers every compilation unit starts with
  std::vector<std::string> kernel_names;
  std::string summary() const;
};

// Builds the plan.  Throws std::runtime_error with a diagnostic on failure.
// With TF32 the attention rewrite runs first; plan.fn then points at the
// rewritten function, which has the same parameters and results as `f`.
Plan build_plan(const Function& f, Precision prec, bool fuse_attention = true);

// Replaces attention regions (and their reverse-mode gradients) by fused
// attention ops.  Returns nullptr when nothing matched (attn_rewrite.cpp).
std::unique_ptr<Function> rewrite_attention(const Function& f, std::string* log);

// Replaces transpose(one_hot(idx, V)) @ adj (+ its batch reduce), Sheaf's
// embedding gradient, by OpKind::ScatterAddRows (embed_grad.cpp).  Returns
// nullptr when nothing matched.
std::unique_ptr<Function> rewrite_embedding_grad(const Function& f, std::string* log);

// Merges sibling GEMMs: dot_generals (or batch-reduced dot_generals) that
// share one operand while their other operands are adjacent blocks of one
// buffer become one wider GEMM whose result the siblings slice; sums of
// dot_generals over adjacent blocks of the contraction become one deeper
// GEMM; and a sum of zero-pads that reassembles a sliced value becomes that
// value.  Returns nullptr when nothing changed (merge_dots.cpp).
std::unique_ptr<Function> merge_sibling_dots(const Function& f, std::string* log);

// Row-major strides of a shape.
std::vector<int64_t> row_major(const std::vector<int64_t>& shape);

// numpy-style no-copy reshape of a strided view; false if impossible.
bool reshape_view(const std::vector<int64_t>& oshape, const std::vector<int64_t>& ostr,
                  const std::vector<int64_t>& nshape, std::vector<int64_t>* nstr);

}  // namespace sb
