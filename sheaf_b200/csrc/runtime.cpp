// Session, buffers, module loading and function execution behind the C ABI.
// Role model: sheaf/src/runtime/iree_session.rs (IreeSession: session creation
// :174, load_vmfb :373, call_device :574), buffer_convert.rs and
// device_buffer.rs.  One CUDA stream per session; all work on a session is
// stream-ordered, so buffers returned by a call may be consumed by the next
// call without a host synchronization.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <functional>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <sstream>
#include <string>
#include <thread>
#include <tuple>
#include <vector>

#include "../../include/sheaf_b200.h"
#include "ir.h"
#include "jit.h"
#include "kernels/kernels.h"
#include "kernels/pdl.h"
#include "nccl_dl.h"
#include "plan.h"

struct sb_status {
  sb_status_code code;
  std::string message;
};

namespace sb {
namespace {

sb_status* make_status(sb_status_code code, const std::string& msg) { return new sb_status{code, msg}; }

sb_status* cuda_status(cudaError_t e, const char* what) {
  sb_status_code code = e == cudaErrorMemoryAllocation ? SB_STATUS_RESOURCE_EXHAUSTED
                        : e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver ? SB_STATUS_UNAVAILABLE
                                                                                       : SB_STATUS_INTERNAL;
  return make_status(code, std::string("CUDA error in ") + what + ": " + cudaGetErrorName(e) + " (" +
                               cudaGetErrorString(e) + ")");
}

#define SB_CUDA(expr)                                   \
  do {                                                  \
    cudaError_t e_ = (expr);                            \
    if (e_ != cudaSuccess) return cuda_status(e_, #expr); \
  } while (0)

bool etype_to_dtype(uint32_t et, DType* out) {
  switch (et) {
    case SB_ELEMENT_TYPE_FLOAT_32: *out = DType::F32; return true;
    case SB_ELEMENT_TYPE_BFLOAT_16: *out = DType::BF16; return true;
    case SB_ELEMENT_TYPE_INT_32: *out = DType::I32; return true;
  }
  return false;
}

uint32_t dtype_to_etype(DType t) {
  switch (t) {
    case DType::F32: return SB_ELEMENT_TYPE_FLOAT_32;
    case DType::BF16: return SB_ELEMENT_TYPE_BFLOAT_16;
    case DType::I32: return SB_ELEMENT_TYPE_INT_32;
    default: return 0;
  }
}

struct Device {
  int ordinal = 0;
  cudaStream_t stream = nullptr;
  // data parallel with SB_SESSION_FLAG_OVERLAP_ALLREDUCE: gradient buckets are
  // all-reduced on comm_stream while the backward continues on `stream`
  cudaStream_t comm_stream = nullptr;
  cudaEvent_t ready = nullptr, reduced = nullptr;
  std::atomic<uint64_t> allocated{0}, freed{0}, live{0}, peak{0};
  void note_alloc(size_t n) {
    allocated += n;
    uint64_t l = (live += n);
    uint64_t p = peak.load();
    while (l > p && !peak.compare_exchange_weak(p, l)) {}
  }
  void note_free(size_t n) {
    freed += n;
    live -= n;
  }
  ~Device() {
    if (comm_stream) {
      cudaSetDevice(ordinal);
      cudaStreamSynchronize(comm_stream);
      cudaStreamDestroy(comm_stream);
      cudaEventDestroy(ready);
      cudaEventDestroy(reduced);
    }
    if (stream) {
      cudaSetDevice(ordinal);
      cudaStreamSynchronize(stream);
      cudaStreamDestroy(stream);
    }
  }
};

}  // namespace
}  // namespace sb

namespace sb {
namespace {
struct OutSlot;
}
}  // namespace sb

struct sb_buffer {
  std::atomic<int> refs{1};
  std::shared_ptr<sb::Device> dev;
  void* ptr = nullptr;
  size_t bytes = 0;
  bool owned = false;
  sb::Type type;
  std::shared_ptr<sb::OutSlot> slot;  // output of a graph replay: memory owned by the slot
};

namespace sb {
namespace {

sb_buffer* new_device_buffer(const std::shared_ptr<Device>& dev, const Type& t, sb_status** st) {
  auto* b = new sb_buffer();
  b->dev = dev;
  b->type = t;
  b->bytes = (size_t)t.numel() * dtype_bytes(t.dtype);
  b->owned = true;
  if (b->bytes) {
    cudaError_t e = cudaMallocAsync(&b->ptr, b->bytes, dev->stream);
    if (e != cudaSuccess) {
      *st = cuda_status(e, "cudaMallocAsync");
      delete b;
      return nullptr;
    }
    dev->note_alloc(b->bytes);
  }
  return b;
}

// One all-reduce of a replayed data-parallel call: a byte range of the slot.
struct Bucket {
  size_t begin = 0, end = 0;
  int32_t op = SB_REDUCE_MEAN;
};

// Output memory of one replayable CUDA graph of a function: every output of a
// call lives in one allocation; the sb_buffers returned by the call share it
// and hand it back (held drops to 0) once they are all released, after which
// the next call can replay the graph into the same memory.
struct OutSlot {
  std::shared_ptr<Device> dev;
  void* base = nullptr;
  std::vector<size_t> off;          // byte offset of each output
  std::atomic<int> held{0};         // outputs of the last replay still referenced
  cudaGraphExec_t exec = nullptr;   // the function's steps, captured with these outputs
  std::vector<void*> direct_in;     // input addresses baked into exec (staged inputs: nullptr)
  uint64_t kernels = 0;             // kernels in exec
  std::vector<Bucket> buckets;      // captured all-reduces (data parallel)
  std::vector<int32_t> reduce_sig;  // per output reduction the graph applies (empty: none)
  ~OutSlot() {
    if (!dev) return;
    cudaSetDevice(dev->ordinal);
    if (exec) cudaGraphExecDestroy(exec);
    if (base) cudaFree(base);
  }
};

struct LoadedFunction {
  std::string qname;
  const Function* fn = nullptr;
  Plan plan;
  std::vector<double> prof_ms;
  std::vector<uint64_t> prof_n;
  std::vector<uint64_t> prof_launches;  // kernels launched by the step (last profiled call)
  std::vector<cudaKernel_t> kern, fin;
  std::map<int, void*> const_ptr;
  void* arena = nullptr;
  size_t arena_cap = 0;
  void* ws = nullptr;
  size_t ws_cap = 0;
  // workspace that holds every deferred split-K partial set of a call at
  // once (the next eager call grows the workspace to it)
  size_t ws_want = 0;
  uint64_t calls = 0;
  // CUDA-graph replay (see run_graph)
  std::vector<std::shared_ptr<OutSlot>> slots;
  std::vector<void*> last_in;      // input addresses of the previous call
  std::vector<char> staged;        // per input: the graph reads a staging copy
  std::vector<void*> stage_buf;    // the staging copies (library-owned)
  bool graphs_off = false;         // capture failed: eager from now on
};

struct LoadedModule {
  std::unique_ptr<Module> mod;
  std::vector<cudaLibrary_t> libs;
  std::vector<std::unique_ptr<LoadedFunction>> fns;
};

struct Nccl {
  ncclComm_t comm = nullptr;
  bool aborted = false;
};

}  // namespace
}  // namespace sb

struct sb_session {
  sb_session_options opts;
  std::shared_ptr<sb::Device> dev;
  std::mutex mu;
  std::vector<std::unique_ptr<sb::LoadedModule>> modules;
  std::map<std::string, sb::LoadedFunction*> by_name;
  std::string cache_dir;
  sb::Nccl nccl;
  bool used_tc = false;  // a tcgen05 GEMM ran on this session
  // per-step CUDA-event timing (sb_session_set_profiling)
  bool profiling = false;
  struct Pending {
    sb::LoadedFunction* fn;
    int step;
    cudaEvent_t a, b;
    uint64_t launches;  // the launch counter at the step's start, then the step's launches
  };
  std::vector<Pending> pending;
  std::vector<cudaEvent_t> free_events;
  cudaEvent_t event() {
    if (!free_events.empty()) {
      cudaEvent_t e = free_events.back();
      free_events.pop_back();
      return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
  }
};

namespace sb {
namespace {

int64_t deadline_ms(const sb_session* s) {
  return s->opts.collective_timeout_ms > 0 ? s->opts.collective_timeout_ms : 600000;
}

// Waits for all work on the session stream with a host deadline.  When NCCL is
// active and the deadline passes, the communicator is aborted so the pending
// collective kernels return, and DEADLINE_EXCEEDED is reported.
sb_status* wait_stream(sb_session* s, int64_t timeout_ms) {
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t e = cudaStreamQuery(s->dev->stream);
    if (e == cudaSuccess) {
      if (s->used_tc) {
        int code = gemm_tcgen05_error();
        if (code)
          return make_status(SB_STATUS_INTERNAL, "tensor-core kernel gave up on a bounded wait (code " +
                                                     std::to_string(code) + "); results are invalid");
      }
      return nullptr;
    }
    if (e != cudaErrorNotReady) return cuda_status(e, "cudaStreamQuery");
    if (s->nccl.comm) {
      ncclResult_t ae = ncclSuccess;
      nccl_api().async_error(s->nccl.comm, &ae);
      if (ae != ncclSuccess && ae != ncclInProgress) {
        nccl_api().comm_abort(s->nccl.comm);
        s->nccl.comm = nullptr;
        s->nccl.aborted = true;
        return make_status(SB_STATUS_INTERNAL, std::string("NCCL error: ") + nccl_api().error_string(ae));
      }
    }
    auto el = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
    if (timeout_ms > 0 && el > timeout_ms) {
      if (s->nccl.comm) {
        nccl_api().comm_abort(s->nccl.comm);
        s->nccl.comm = nullptr;
        s->nccl.aborted = true;
      }
      return make_status(SB_STATUS_DEADLINE_EXCEEDED,
                         "device work did not finish within " + std::to_string(timeout_ms) + " ms");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// The communicator is nonblocking: after ncclGroupEnd returns ncclInProgress the
// collectives are enqueued onto the stream by NCCL in the background, and the
// communicator accepts no new call until ncclCommGetAsyncError stops reporting
// ncclInProgress.  Polls that state with the collective deadline; on error or
// timeout the communicator is aborted.
sb_status* nccl_settle(sb_session* s) {
  const NcclApi& api = nccl_api();
  auto t0 = std::chrono::steady_clock::now();
  int64_t tmo = deadline_ms(s);
  for (;;) {
    ncclResult_t ae = ncclInProgress;
    api.async_error(s->nccl.comm, &ae);
    if (ae == ncclSuccess) return nullptr;
    bool late = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count() > tmo;
    if (ae != ncclInProgress || late) {
      api.comm_abort(s->nccl.comm);
      s->nccl.comm = nullptr;
      s->nccl.aborted = true;
      if (late) return make_status(SB_STATUS_DEADLINE_EXCEEDED, "NCCL collective was not enqueued within the deadline");
      return make_status(SB_STATUS_INTERNAL, std::string("NCCL error: ") + api.error_string(ae));
    }
    std::this_thread::yield();
  }
}

sb_status* load_module(sb_session* s, const std::string& text, const Prebuilt* prebuilt = nullptr) {
  std::string err;
  auto mod = parse_module(text, &err);
  if (!mod) return make_status(SB_STATUS_INVALID_ARGUMENT, err);
  auto lm = std::make_unique<LoadedModule>();
  std::vector<std::string> snippets;
  Precision prec = (Precision)s->opts.precision;
  for (auto& f : mod->funcs) {
    auto lf = std::make_unique<LoadedFunction>();
    lf->fn = &f;
    lf->qname = mod->name.empty() ? f.name : mod->name + "." + f.name;
    try {
      lf->plan = build_plan(f, prec, !(s->opts.flags & SB_SESSION_FLAG_NO_ATTENTION_FUSION));
    } catch (const std::exception& e) {
      return make_status(SB_STATUS_UNIMPLEMENTED, "planning @" + f.name + ": " + e.what());
    }
    for (auto& sn : lf->plan.snippets) snippets.push_back(sn);
    lm->fns.push_back(std::move(lf));
  }
  // Kernel names are per function (k0, k1, ...): prefix them per function.
  // (build_plan names kernels from 0 for each function, so compile per function.)
  std::map<std::string, cudaKernel_t> kernels;
  SB_CUDA(cudaSetDevice(s->dev->ordinal));
  for (size_t fi = 0; fi < lm->fns.size(); ++fi) {
    auto& lf = lm->fns[fi];
    std::vector<CubinChunk> chunks = split_source(lf->plan.snippets, lf->plan.prelude, 16);
    try {
      if (!lf->plan.snippets.empty()) compile_chunks(chunks, s->cache_dir, prebuilt);
    } catch (const std::exception& e) {
      return make_status(SB_STATUS_INTERNAL, "kernel compilation for @" + lf->fn->name + " failed: " + e.what());
    }
    std::vector<cudaLibrary_t> libs;
    if (!lf->plan.snippets.empty()) {
      for (auto& ch : chunks) {
        cudaLibrary_t lib;
        SB_CUDA(cudaLibraryLoadData(&lib, ch.cubin.data(), nullptr, nullptr, 0, nullptr, nullptr, 0));
        libs.push_back(lib);
        lm->libs.push_back(lib);
      }
    }
    auto find = [&](const std::string& name, cudaKernel_t* k) -> bool {
      for (auto lib : libs) {
        if (cudaLibraryGetKernel(k, lib, name.c_str()) == cudaSuccess) return true;
        cudaGetLastError();  // a miss in one chunk is expected; do not leave it sticky
      }
      return false;
    };
    for (auto& st : lf->plan.steps) {
      cudaKernel_t k = nullptr, fk = nullptr;
      if (!st.kernel.empty() && !find(st.kernel, &k))
        return make_status(SB_STATUS_INTERNAL, "generated kernel " + st.kernel + " not found");
      if (!st.finish_kernel.empty() && !find(st.finish_kernel, &fk))
        return make_status(SB_STATUS_INTERNAL, "generated kernel " + st.finish_kernel + " not found");
      lf->kern.push_back(k);
      lf->fin.push_back(fk);
    }
    // dense constants
    for (int v : lf->plan.constants) {
      const Op& op = lf->plan.fn->ops[lf->plan.fn->producer[v]];
      size_t n = (size_t)op.type.numel();
      std::vector<uint8_t> host(n * dtype_bytes(op.type.dtype));
      for (size_t i = 0; i < n; ++i) {
        double x = op.values[i];
        switch (op.type.dtype) {
          case DType::F32: { float f = (float)x; std::memcpy(&host[i * 4], &f, 4); break; }
          case DType::I32: { int32_t q = (int32_t)x; std::memcpy(&host[i * 4], &q, 4); break; }
          case DType::I1: host[i] = x != 0; break;
          default: return make_status(SB_STATUS_UNIMPLEMENTED, "constant element type");
        }
      }
      void* p = nullptr;
      SB_CUDA(cudaMalloc(&p, std::max<size_t>(host.size(), 4)));
      SB_CUDA(cudaMemcpy(p, host.data(), host.size(), cudaMemcpyHostToDevice));
      lf->const_ptr[v] = p;
    }
    if (lf->plan.arena_bytes) {
      SB_CUDA(cudaMalloc(&lf->arena, (size_t)lf->plan.arena_bytes));
      lf->arena_cap = (size_t)lf->plan.arena_bytes;
    }
  }
  lm->mod = std::move(mod);
  for (auto& lf : lm->fns) {
    s->by_name[lf->qname] = lf.get();
    if (!s->by_name.count(lf->fn->name)) s->by_name[lf->fn->name] = lf.get();
  }
  s->modules.push_back(std::move(lm));
  return nullptr;
}

// Kernel name of a step as the profile report and plan listing show it.
std::string step_name(const Step& st) {
  if (st.kind == StepKind::Gemm) return "gemm";
  if (st.kind == StepKind::Sort) return "sort";
  if (st.kind == StepKind::Convert) return "operand_shadow";
  if (st.kind == StepKind::Scatter) return "scatter_add_rows";
  if (st.kind == StepKind::Attn)
    return st.attn.kind == OpKind::AttnFwd ? "attn_fwd" : "attn_bwd";
  return st.kernel;
}

sb_status* launch_generated(cudaKernel_t k, const std::vector<const void*>& ptrs, int64_t gx, int64_t gy,
                            int64_t block, cudaStream_t stream) {
  void* args[1] = {(void*)ptrs.data()};
  // generated kernels start with griddepcontrol.wait: they may be launched
  // while the previous kernel drains (programmatic dependent launch)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)gx, (unsigned)gy, 1);
  cfg.blockDim = dim3((unsigned)block);
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  launch_counter().fetch_add(1, std::memory_order_relaxed);
  SB_CUDA(cudaLaunchKernelExC(&cfg, (const void*)k, args));
  return nullptr;
}

// SHEAF_B200_GEMM_PAIRS=0: every GEMM step in its own launch (for
// comparisons; pairing changes no result, since a product's summation order
// depends only on its shape).
bool gemm_pairs_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("SHEAF_B200_GEMM_PAIRS");
    return !(e && std::string(e) == "0");
  }();
  return on;
}

// Enqueues a call's work on `stream`: TF32 copies of parameters, every plan
// step, and the copies of outputs that no step writes (to outp[j]).  ptr holds
// the device address of every materialized value.  before(si, flush), if set,
// runs before step si is enqueued (the data-parallel bucket flushes); it must
// call flush() before a collective reads step outputs, so that deferred
// split-K reductions are done.  capturing: the stream is being captured into
// a graph, so nothing may allocate.
//
// Split-K reductions of GEMM steps are deferred and launched together (one
// launch for up to kReduceSegments of them) when a step reads one of their
// outputs, when the workspace is full, before a collective, and at the end:
// the weight-gradient GEMMs of a backward pass, whose outputs no later step
// reads, share one reduction launch.  Their partial sums stay in disjoint
// parts of the workspace until then.  Profiled calls reduce right away, so
// that every step's time includes its own reduction.
//
// Two consecutive GEMM steps, the second not reading the first's result,
// run as one tensor-core launch (gemm_pair) where both allow it; profiled
// calls launch every step on its own.
using BeforeStep = std::function<sb_status*(size_t, const std::function<sb_status*()>&)>;
sb_status* enqueue_steps(sb_session* s, LoadedFunction* lf, std::vector<void*>& ptr, const std::vector<void*>& outp,
                         const BeforeStep& before, bool capturing) {
  const Function& f = *lf->plan.fn;
  const Plan& plan = lf->plan;
  cudaStream_t stream = s->dev->stream;
  // TF32-rounded copies of parameters read by tensor-core GEMMs
  // (kRoundSegments weights per launch: one launch for a typical model)
  std::map<int, const float*> rounded;
  RoundSegments segs{};
  for (size_t j = 0; j < plan.rounded_params.size(); ++j) {
    int v = plan.rounded_params[j];
    float* dst = (float*)((char*)lf->arena + plan.rounded_offset[j]);
    segs.src[segs.count] = (const float*)ptr[v];
    segs.dst[segs.count] = dst;
    segs.n[segs.count] = f.value_types[v].numel();
    if (++segs.count == kRoundSegments || j + 1 == plan.rounded_params.size()) {
      cudaError_t e = round_tf32_segments(segs, stream);
      if (e != cudaSuccess) { return cuda_status(e, "round_tf32_segments"); }
      segs.count = 0;
    }
    rounded[v] = dst;
  }
  ReduceSegments red;
  std::vector<int> red_vals;  // values the pending reductions write
  size_t ws_off = 0;          // workspace bytes held by pending partial sums
  size_t ws_run = 0;          // the same, not counting flushes forced by a full workspace
  const bool defer = !s->profiling;
  ColSums cols;  // deferred finishes of row-group column sums
  Bf16Segments cvt{};  // consecutive bf16 operand-shadow conversions
  const std::function<sb_status*()> flush_red = [&]() -> sb_status* {
    if (red.count) {
      cudaError_t e = splitk_reduce_segments(red, stream);
      if (e != cudaSuccess) return cuda_status(e, "splitk_reduce_segments");
      red.count = 0;
    }
    if (cols.count) {
      cudaError_t e = col_sum_segments(cols, stream);
      if (e != cudaSuccess) return cuda_status(e, "col_sum_segments");
      cols.count = 0;
    }
    red_vals.clear();
    ws_off = 0;
    return nullptr;
  };
  // the GEMM of step st: operand addresses (view offsets count elements of
  // the buffer read: f32, or bf16 for bf16 operands and bf16 shadows)
  auto gemm_args = [&](const Step& st) {
    const GemmDesc& g = st.gemm;
    GemmArgs a;
    auto operand = [&](const View& w, bool rnd, int shadow) -> const float* {
      const int64_t es = g.bf16 ? 2 : 4;
      if (shadow >= 0) return (const float*)((char*)lf->arena + plan.shadows[shadow].offset + w.offset * es);
      const char* base = rnd ? (const char*)rounded[w.value] : (const char*)ptr[w.value];
      return (const float*)(base + w.offset * es);
    };
    a.a = operand(g.a, g.a_rounded, g.a_shadow);
    a.b = operand(g.b, g.b_rounded, g.b_shadow);
    a.bf16 = g.bf16 ? 1 : 0;
    a.c = (float*)ptr[st.root];
    a.round_out = g.round_out ? 1 : 0;
    a.batch = g.batch; a.M = g.M; a.N = g.N; a.K = g.K;
    a.sab = g.sab; a.sam = g.sam; a.sak = g.sak;
    a.sbb = g.sbb; a.sbk = g.sbk; a.sbn = g.sbn;
    a.scb = g.M * g.N; a.scm = g.N; a.scn = 1;
    if (g.epi) {
      a.epi = g.epi;
      a.c2 = (float*)ptr[st.extra_roots[0]];
      a.round_out2 = g.round_out2 ? 1 : 0;
    }
    return a;
  };
  std::vector<const void*> args;
  for (size_t si = 0; si < plan.steps.size(); ++si) {
    if (before)
      if (sb_status* e = before(si, flush_red)) return e;
    const Step& st = plan.steps[si];
    if (!red_vals.empty()) {
      bool reads = false;
      for (int l : st.leaves) reads |= std::find(red_vals.begin(), red_vals.end(), l) != red_vals.end();
      if (reads) {
        if (sb_status* e = flush_red()) return e;
        ws_run = 0;
      }
    }
    if (!ptr[st.root] && st.elements) { return make_status(SB_STATUS_INTERNAL, "unplaced value"); }
    cudaEvent_t ev_a = nullptr, ev_b = nullptr;
    if (s->profiling) {
      ev_a = s->event();
      ev_b = s->event();
      cudaEventRecord(ev_a, stream);
      s->pending.push_back({lf, (int)si, ev_a, ev_b, launch_counter().load()});
    }
    struct EndEvent {
      cudaEvent_t e;
      cudaStream_t s;
      sb_session* ss;
      ~EndEvent() {
        if (!e) return;
        cudaEventRecord(e, s);
        auto& p = ss->pending.back();
        p.launches = launch_counter().load() - p.launches;
      }
    } end_event{ev_b, stream, s};
    if (st.kind == StepKind::Convert) {
      const Shadow& sh = plan.shadows[st.shadow];
      char* dst = (char*)lf->arena + sh.offset;
      const float* src = (const float*)ptr[sh.value];
      if (defer && sh.dtype == DType::BF16) {
        // consecutive bf16 conversions (the weights' copies at the start of
        // a call) go out as one launch
        cvt.src[cvt.count] = src;
        cvt.dst[cvt.count] = (uint16_t*)dst;
        cvt.n[cvt.count] = st.elements;
        ++cvt.count;
        const bool more = si + 1 < plan.steps.size() && plan.steps[si + 1].kind == StepKind::Convert &&
                          plan.shadows[plan.steps[si + 1].shadow].dtype == DType::BF16;
        if (!more || cvt.count == kRoundSegments) {
          cudaError_t e = bf16_segments(cvt, stream);
          cvt.count = 0;
          if (e != cudaSuccess) { return cuda_status(e, "operand shadows"); }
        }
        continue;
      }
      cudaError_t e = sh.dtype == DType::BF16 ? bf16_copy(src, (uint16_t*)dst, st.elements, stream)
                                              : round_tf32_copy(src, (float*)dst, st.elements, stream);
      if (e != cudaSuccess) { return cuda_status(e, "operand shadow"); }
      continue;
    }
    if (st.kind == StepKind::Gemm) {
      GemmArgs a = gemm_args(st);
      // the next step, a GEMM that does not read this one's result, shares the
      // launch (a layer's dX and dW in a backward pass)
      if (defer && gemm_pairs_enabled() && si + 1 < plan.steps.size() && plan.steps[si + 1].kind == StepKind::Gemm &&
          !st.gemm.epi && !plan.steps[si + 1].gemm.epi) {
        const Step& nx = plan.steps[si + 1];
        const bool indep = std::find(nx.leaves.begin(), nx.leaves.end(), st.root) == nx.leaves.end();
        GemmArgs ab[2] = {a, gemm_args(nx)};
        const size_t n0 = (gemm_workspace(ab[0], s->opts.precision) + 255) & ~(size_t)255;
        const size_t n1 = (gemm_workspace(ab[1], s->opts.precision) + 255) & ~(size_t)255;
        if (indep && !(capturing && n0 + n1 > lf->ws_cap)) {
          bool reads = false;
          for (int l : nx.leaves) reads |= std::find(red_vals.begin(), red_vals.end(), l) != red_vals.end();
          if (reads || red.count + 2 > kReduceSegments || ws_off + n0 + n1 > lf->ws_cap) {
            if (sb_status* e = flush_red()) return e;
            if (reads) ws_run = 0;
          }
          if (n0 + n1 > lf->ws_cap) {
            if (lf->ws) cudaFreeAsync(lf->ws, stream);
            if (cudaMallocAsync(&lf->ws, n0 + n1, stream) != cudaSuccess) { lf->ws = nullptr; lf->ws_cap = 0; }
            else lf->ws_cap = n0 + n1;
          }
          SplitReduce d2[2];
          cudaError_t e = gemm_pair(ab, s->opts.precision, lf->ws ? (char*)lf->ws + ws_off : nullptr,
                                    lf->ws ? lf->ws_cap - ws_off : 0, stream, d2);
          if (e == cudaSuccess) {
            s->used_tc = true;
            const int roots[2] = {st.root, nx.root};
            for (int q = 0; q < 2; ++q)
              if (d2[q].splits > 0) {
                red.seg[red.count++] = d2[q];
                red_vals.push_back(roots[q]);
              }
            ws_off += n0 + n1;
            ws_run += n0 + n1;
            lf->ws_want = std::max(lf->ws_want, ws_run);
            if (red.count == kReduceSegments)
              if (sb_status* e2 = flush_red()) return e2;
            ++si;  // the next step ran in this launch; its collectives are due now
            if (before)
              if (sb_status* e2 = before(si, flush_red)) return e2;
            continue;
          }
          if (e != cudaErrorNotSupported) return cuda_status(e, "gemm pair");
        }
      }
      const size_t need = (gemm_workspace(a, s->opts.precision) + 255) & ~(size_t)255;
      if (ws_off + need > lf->ws_cap)
        if (sb_status* e = flush_red()) return e;  // the pending partials' space is free again
      // a stream being captured into a graph must not allocate: the eager
      // call that precedes every capture sized the workspace
      if (need > lf->ws_cap && capturing) return make_status(SB_STATUS_UNAVAILABLE, "workspace grows during capture");
      if (need > lf->ws_cap) {
        if (lf->ws) cudaFreeAsync(lf->ws, stream);
        if (cudaMallocAsync(&lf->ws, need, stream) != cudaSuccess) { lf->ws = nullptr; lf->ws_cap = 0; }
        else lf->ws_cap = need;
      }
      bool tc = false;
      SplitReduce d;
      cudaError_t e = gemm(a, s->opts.precision, lf->ws ? (char*)lf->ws + ws_off : nullptr,
                           lf->ws ? lf->ws_cap - ws_off : 0, stream, &tc, defer ? &d : nullptr);
      if (tc) s->used_tc = true;
      if (e != cudaSuccess) { return cuda_status(e, "gemm"); }
      if (defer && d.splits > 0) {
        red.seg[red.count++] = d;
        red_vals.push_back(st.root);
        ws_off += need;
        ws_run += need;
        lf->ws_want = std::max(lf->ws_want, ws_run);
        if (red.count == kReduceSegments)
          if (sb_status* e2 = flush_red()) return e2;
      }
      continue;
    }
    if (st.kind == StepKind::Scatter) {
      const bool f32 = f.value_types[st.leaves[0]].dtype == DType::F32;
      cudaError_t e = scatter_add_rows(ptr[st.leaves[0]], f32, (const float*)ptr[st.leaves[1]], (float*)ptr[st.root],
                                       st.gemm.K, st.gemm.N, st.gemm.M, (char*)lf->arena + plan.scratch_offset[si],
                                       stream);
      s->used_tc = true;  // its bounds checks report through the same error word
      if (e != cudaSuccess) { return cuda_status(e, "scatter_add_rows"); }
      continue;
    }
    if (st.kind == StepKind::Sort) {
      cudaError_t e = sort_pairs((const float*)ptr[st.leaves[0]], (const int*)ptr[st.leaves[1]], (float*)ptr[st.root],
                                 st.gemm.M, st.gemm.N, st.gemm.K != 0, stream);
      if (e != cudaSuccess) { return cuda_status(e, "sort"); }
      continue;
    }
    if (st.kind == StepKind::Attn) {
      const AttnDesc& d = st.attn;
      AttnArgs a;
      a.kind = AttnKind::Fwd;
      a.B = d.B; a.H = d.H; a.T = d.T; a.hd = 64;
      a.scale = (float)d.scale;
      a.causal = d.causal;
      a.round_out = d.round_out;
      a.out = (float*)ptr[st.root];
      auto view = [&](size_t i) {
        const View& w = d.in[i];
        AttnView r;
        r.p = (d.rounded[i] ? rounded[w.value] : (const float*)ptr[w.value]) + w.offset;
        r.sb = w.strides[0]; r.sh = w.strides[1]; r.st = w.strides[2];
        return r;
      };
      a.q = view(0); a.k = view(1); a.v = view(2);
      cudaError_t e = cudaSuccess;
      if (d.kind == OpKind::AttnFwd) {
        e = attention(a, stream);
      } else {
        // [dQ, dK, dV as (B,T,3,H,64) | D (B,H,T)]: the dQ pass writes dQ
        // and D, the dK/dV pass reads D
        const int64_t hd = d.H * 64, n = d.B * d.T * hd;
        float* base = (float*)ptr[st.root];
        const View& l = d.in[5];
        a.dy = view(3);
        a.y = view(4);
        a.lse = (const float*)ptr[l.value] + l.offset;
        a.l_sb = l.strides[0]; a.l_sh = l.strides[1]; a.l_st = l.strides[2];
        a.out_ld = 3 * hd;
        a.stats = base + 3 * n;
        a.kind = AttnKind::BwdQ;
        a.out = base;
        e = attention(a, stream);
        if (e == cudaSuccess) {
          a.kind = AttnKind::BwdKV;
          a.dsum = base + 3 * n;
          a.d_sb = d.H * d.T; a.d_sh = d.T; a.d_st = 1;
          a.out = base + hd;
          a.out_v = base + 2 * hd;
          a.stats = nullptr;
          e = attention(a, stream);
        }
      }
      s->used_tc = true;
      if (e != cudaSuccess) { return cuda_status(e, "attention"); }
      continue;
    }
    args.clear();
    for (int l : st.leaves) args.push_back(ptr[l]);
    args.push_back(ptr[st.root]);
    for (int e : st.extra_roots) args.push_back(ptr[e]);
    void* scratch = nullptr;
    if (st.splits > 1) {
      scratch = (char*)lf->arena + plan.scratch_offset[si];
      args.push_back(scratch);
    }
    for (int k : st.shadow_outs) args.push_back((char*)lf->arena + plan.shadows[k].offset);
    sb_status* e = launch_generated(lf->kern[si], args, st.grid, st.grid_y, st.block, stream);
    if (e) { return e; }
    if (st.splits > 1) {
      if (defer && st.finish_deferred && (int)st.col_finish.size() <= kColSegments) {
        // column sums no later step reads: added with other steps' at the next flush
        if (cols.count + (int)st.col_finish.size() > kColSegments)
          if (sb_status* e2 = flush_red()) return e2;
        for (const Step::ColFinish& cf : st.col_finish) {
          const int v = cf.out == 0 ? st.root : st.extra_roots[cf.out - 1];
          ColSum& c = cols.seg[cols.count++];
          c.s = (const float*)scratch + cf.offset;
          c.out = (float*)ptr[v];
          c.C = (int)st.col_C;
          c.parts = (int)st.splits;
          red_vals.push_back(v);
        }
        continue;
      }
      e = launch_generated(lf->fin[si], args, st.finish_grid, 1, st.block, stream);
      if (e) { return e; }
    }
  }
  if (sb_status* e = flush_red()) return e;
  // room for every deferred partial set of a call, for the calls that follow
  // (a captured call cannot allocate)
  if (!capturing && lf->ws_want > lf->ws_cap) {
    if (lf->ws) cudaFreeAsync(lf->ws, stream);
    if (cudaMallocAsync(&lf->ws, lf->ws_want, stream) != cudaSuccess) { lf->ws = nullptr; lf->ws_cap = 0; }
    else lf->ws_cap = lf->ws_want;
  }
  // outputs not written by a step: copies
  for (size_t j = 0; j < f.returns.size(); ++j) {
    if (plan.output_step[j] >= 0) continue;
    int v = f.returns[j];
    const size_t bytes = (size_t)f.value_types[v].numel() * dtype_bytes(f.value_types[v].dtype);
    if (bytes && ptr[v]) SB_CUDA(cudaMemcpyAsync(outp[j], ptr[v], bytes, cudaMemcpyDeviceToDevice, stream));
  }
  return nullptr;
}

// CUDA-graph replay of a function.  Launching ~150-300 kernels per call costs
// the host milliseconds (tensor-map encoding, launch calls), as much as the
// GPU needs for the step itself at small batch.  From the second call on, the
// function's steps are captured once into a graph and replayed: one launch per
// call.  A graph bakes in addresses, so
//  * outputs go to library-owned slots (OutSlot): a replay needs a slot whose
//    outputs the caller has released; up to kMaxSlots slots are kept;
//  * inputs whose address changed since the previous call (a new token batch
//    each step) are "staged": the graph reads a library-owned copy, refreshed
//    by one device-to-device copy per call; inputs at a stable address (the
//    resident parameters) are read in place, and a change of one of them
//    recaptures the slot's graph.
// The first call runs eagerly (it also picks the GEMM tile configurations and
// sizes the workspace), so capture never allocates.  Data-parallel calls with
// a reduction and profiled calls always run eagerly.  *used = false: the
// caller runs the call eagerly.
constexpr int kMaxSlots = 4;
constexpr size_t kMaxStagedBytes = 64u << 20;

// SHEAF_B200_GRAPH_LOG=1: one stderr line per call saying how it ran
// (captured, replayed, or eager and why).
bool graph_log_on() {
  static const bool on = [] {
    const char* e = std::getenv("SHEAF_B200_GRAPH_LOG");
    return e && std::string(e) == "1";
  }();
  return on;
}

void graph_log(const LoadedFunction* lf, const std::string& what) {
  if (graph_log_on()) std::fprintf(stderr, "sheaf_b200: @%s: %s\n", lf->qname.c_str(), what.c_str());
}

bool graphs_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("SHEAF_B200_GRAPHS");
    return !(e && std::string(e) == "0");
  }();
  return on;
}

// Data-parallel calls: the gradient all-reduce is captured into the graph too.
// The outputs are laid out in the order in which the backward completes them,
// so that a bucket of outputs is one contiguous byte range of the slot and
// takes a single ncclAllReduce (on the comm stream, overlapped with the rest
// of the backward when the session overlaps); the replay issues no NCCL call
// from the host.

sb_status* capture_reductions(sb_session* s, LoadedFunction* lf, const int32_t* reduce, OutSlot* slot,
                              std::vector<void*>& ptr, const std::vector<void*>& outp);

// Step after which output j is complete and read by no later step (outputs
// copied after the steps, and values returned more than once: past the end).
std::vector<int> ready_steps(const LoadedFunction* lf) {
  const Function& f = *lf->plan.fn;
  const Plan& plan = lf->plan;
  std::vector<int> last(f.num_values(), -1);
  for (int si = 0; si < (int)plan.steps.size(); ++si)
    for (int l : plan.steps[si].leaves) last[l] = si;
  std::vector<int> times(f.num_values(), 0);
  for (int v : f.returns) ++times[v];
  std::vector<int> r(f.returns.size());
  for (size_t j = 0; j < f.returns.size(); ++j) {
    const int v = f.returns[j];
    r[j] = (plan.output_step[j] < 0 || times[v] > 1) ? (int)plan.steps.size()
                                                     : std::max(plan.output_step[j], last[v]);
  }
  return r;
}

// Byte layout order of a slot's outputs: with reductions, the reduced outputs
// by the step that completes them (then by reduction), the others after.
std::vector<int> output_order(const LoadedFunction* lf, const int32_t* reduce) {
  const size_t n = lf->plan.fn->returns.size();
  std::vector<int> order(n);
  for (size_t j = 0; j < n; ++j) order[j] = (int)j;
  if (!reduce) return order;
  const std::vector<int> ready = ready_steps(lf);
  auto key = [&](int j) {
    const bool red = reduce[j] != SB_REDUCE_NONE;
    return std::make_tuple(red ? 0 : 1, red ? ready[j] : 0, red ? reduce[j] : 0, j);
  };
  std::sort(order.begin(), order.end(), [&](int a, int b) { return key(a) < key(b); });
  return order;
}

sb_status* capture_reductions(sb_session* s, LoadedFunction* lf, const int32_t* reduce, OutSlot* slot,
                              std::vector<void*>& ptr, const std::vector<void*>& outp) {
  const Function& f = *lf->plan.fn;
  const Plan& plan = lf->plan;
  cudaStream_t stream = s->dev->stream;
  const bool overlap = s->dev->comm_stream != nullptr;
  cudaStream_t cs = overlap ? s->dev->comm_stream : stream;
  for (size_t j = 0; j < f.returns.size(); ++j)
    if (reduce[j] != SB_REDUCE_NONE && f.value_types[f.returns[j]].dtype != DType::F32)
      return make_status(SB_STATUS_UNIMPLEMENTED, "reduce of non-f32 output");
  if (!s->nccl.comm) return make_status(SB_STATUS_FAILED_PRECONDITION, "NCCL communicator is not available");
  // 16 MB buckets: on 2 B200s the nanoGPT step measured 3.31 / 3.27 / 3.23 /
  // 3.16 ms with 2 / 4 / 8 / 16 MB (fewer, larger all-reduces cost less than
  // the overlap that smaller ones would add)
  size_t bucket_limit = 16u << 20;
  if (const char* bb = std::getenv("SHEAF_B200_ALLREDUCE_BUCKET_BYTES"))
    if (std::atoll(bb) > 0) bucket_limit = (size_t)std::atoll(bb);
  const std::vector<int> ready = ready_steps(lf);
  const std::vector<int> order = output_order(lf, reduce);
  // outputs of one bucket are adjacent in `order`, hence in the slot
  size_t next = 0;  // position in `order` of the first output not yet queued
  Bucket cur;
  bool open = false, forked = false;
  auto bytes_of = [&](int j) {
    const int v = f.returns[j];
    return ((size_t)f.value_types[v].numel() * 4 + 255) & ~size_t(255);
  };
  const std::function<sb_status*()>* red_flush = nullptr;  // deferred split-K reductions (during the steps)
  auto flush = [&]() -> sb_status* {
    if (!open) return nullptr;
    open = false;
    if (red_flush)
      if (sb_status* st = (*red_flush)()) return st;
    if (overlap) {
      SB_CUDA(cudaEventRecord(s->dev->ready, stream));
      SB_CUDA(cudaStreamWaitEvent(cs, s->dev->ready, 0));
      forked = true;
    }
    const NcclApi& api = nccl_api();
    char* base = (char*)slot->base;
    ncclResult_t r = api.all_reduce(base + cur.begin, base + cur.begin, (cur.end - cur.begin) / 4, ncclFloat32,
                                    cur.op == SB_REDUCE_MEAN ? ncclAvg : ncclSum, s->nccl.comm, cs);
    if (r != ncclSuccess && r != ncclInProgress)
      return make_status(SB_STATUS_INTERNAL, std::string("ncclAllReduce: ") + api.error_string(r));
    slot->buckets.push_back(cur);
    return nccl_settle(s);
  };
  // queue the reduced outputs completed by step `upto` (inclusive)
  auto queue = [&](int upto) -> sb_status* {
    while (next < order.size()) {
      const int j = order[next];
      if (reduce[j] == SB_REDUCE_NONE || ready[j] > upto) break;
      const size_t b = slot->off[j], e = b + bytes_of(j);
      if (open && (reduce[j] != cur.op || b != cur.end))
        if (sb_status* st = flush()) return st;
      if (!open) {
        cur.begin = b;
        cur.end = b;
        cur.op = reduce[j];
        open = true;
      }
      cur.end = e;
      ++next;
      if (overlap && cur.end - cur.begin >= bucket_limit)
        if (sb_status* st = flush()) return st;
    }
    return nullptr;
  };
  slot->buckets.clear();
  const BeforeStep before = [&](size_t si, const std::function<sb_status*()>& fl) -> sb_status* {
    red_flush = &fl;
    return (overlap && si > 0) ? queue((int)si - 1) : nullptr;
  };
  sb_status* est = enqueue_steps(s, lf, ptr, outp, before, true);
  red_flush = nullptr;
  if (est) return est;
  if (sb_status* st = queue((int)plan.steps.size())) return st;
  if (sb_status* st = flush()) return st;
  if (overlap && forked) {
    SB_CUDA(cudaEventRecord(s->dev->reduced, cs));
    SB_CUDA(cudaStreamWaitEvent(stream, s->dev->reduced, 0));
  }
  return nullptr;
}

sb_status* run_graph(sb_session* s, LoadedFunction* lf, sb_buffer* const* in, size_t nin, const int32_t* reduce,
                     sb_buffer** out, size_t* nout, bool* used) {
  *used = false;
  const Function& f = *lf->plan.fn;
  const Plan& plan = lf->plan;
  cudaStream_t stream = s->dev->stream;
  const bool first = lf->calls == 0;
  bool dp = false;
  if (reduce && s->opts.world_size > 1)
    for (size_t j = 0; j < f.returns.size(); ++j) dp = dp || reduce[j] != SB_REDUCE_NONE;
  if (lf->last_in.size() != nin) {
    lf->last_in.assign(nin, nullptr);
    lf->staged.assign(nin, 0);
    lf->stage_buf.assign(nin, nullptr);
  }
  // inputs that moved since the previous call are staged from now on
  bool restage = false;
  for (size_t i = 0; i < nin; ++i) {
    if (!first && !lf->staged[i] && in[i]->ptr != lf->last_in[i] && in[i]->bytes <= kMaxStagedBytes) {
      lf->staged[i] = 1;
      restage = true;
    }
    lf->last_in[i] = in[i]->ptr;
  }
  if (first) {  // eager: tunes the GEMMs, sizes the workspace
    graph_log(lf, "eager (first call)");
    return nullptr;
  }
  if (restage)                // graphs captured before read those inputs in place
    for (auto& sl : lf->slots)
      if (sl->exec) {
        cudaGraphExecDestroy(sl->exec);
        sl->exec = nullptr;
      }
  for (size_t i = 0; i < nin; ++i)
    if (lf->staged[i] && !lf->stage_buf[i] && in[i]->bytes)
      SB_CUDA(cudaMalloc(&lf->stage_buf[i], in[i]->bytes));
  // a slot whose outputs are free, preferring one whose graph reads these inputs
  std::vector<void*> direct(nin, nullptr);
  for (size_t i = 0; i < nin; ++i)
    if (!lf->staged[i]) direct[i] = in[i]->ptr;
  // slots are laid out and captured for one reduction signature
  std::vector<int32_t> sig;
  if (dp) sig.assign(reduce, reduce + f.returns.size());
  std::shared_ptr<OutSlot> slot;
  for (auto& sl : lf->slots)
    if (sl->held.load() == 0 && sl->reduce_sig == sig && sl->exec && sl->direct_in == direct) { slot = sl; break; }
  if (!slot)
    for (auto& sl : lf->slots)
      if (sl->held.load() == 0 && sl->reduce_sig == sig) { slot = sl; break; }
  if (!slot) {
    if ((int)lf->slots.size() >= kMaxSlots) {
      graph_log(lf, "eager (every output set is held)");
      return nullptr;
    }
    auto sl = std::make_shared<OutSlot>();
    sl->dev = s->dev;
    sl->reduce_sig = sig;
    size_t total = 0;
    sl->off.assign(f.returns.size(), 0);
    for (int jj : output_order(lf, dp ? reduce : nullptr)) {
      const int v = f.returns[jj];
      sl->off[jj] = total;
      total += ((size_t)f.value_types[v].numel() * dtype_bytes(f.value_types[v].dtype) + 255) & ~size_t(255);
    }
    if (total) SB_CUDA(cudaMalloc(&sl->base, total));
    lf->slots.push_back(sl);
    slot = sl;
  }
  std::vector<void*> outp(f.returns.size());
  for (size_t j = 0; j < outp.size(); ++j) outp[j] = (char*)slot->base + slot->off[j];
  if (!slot->exec || slot->direct_in != direct) {
    if (slot->exec) {
      cudaGraphExecDestroy(slot->exec);
      slot->exec = nullptr;
    }
    std::vector<void*> ptr(f.num_values(), nullptr);
    for (size_t i = 0; i < nin; ++i) ptr[i] = lf->staged[i] ? lf->stage_buf[i] : in[i]->ptr;
    for (auto& [v, p] : lf->const_ptr) ptr[v] = p;
    for (size_t j = 0; j < f.returns.size(); ++j)
      if (plan.output_step[j] >= 0) ptr[f.returns[j]] = outp[j];
    for (int v : plan.materialized)
      if (!ptr[v] && plan.value_offset[v] >= 0) ptr[v] = (char*)lf->arena + plan.value_offset[v];
    SB_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
    const uint64_t k0 = launch_counter().load();
    sb_status* st = dp ? capture_reductions(s, lf, reduce, slot.get(), ptr, outp)
                       : enqueue_steps(s, lf, ptr, outp, nullptr, true);
    // kernels recorded into the graph (counted by the launch paths; taken
    // back off the counter, which counts kernels that run)
    slot->kernels = launch_counter().load() - k0;
    launch_counter().fetch_sub(slot->kernels, std::memory_order_relaxed);
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamEndCapture(stream, &graph);
    if (!st && e == cudaSuccess) e = cudaGraphInstantiate(&slot->exec, graph, 0);
    if (graph) cudaGraphDestroy(graph);
    if (st || e != cudaSuccess) {
      slot->exec = nullptr;
      if (dp) {
        // every rank must issue the same collectives: no silent fallback to
        // the eager path's per-leaf all-reduces
        if (st) return st;
        return cuda_status(e, "capturing a data-parallel call");
      }
      // not capturable (e.g. the workspace would have to grow): eager from now on
      std::fprintf(stderr, "sheaf_b200: @%s is not captured into a CUDA graph (%s); its calls run eagerly\n",
                   lf->qname.c_str(), st ? sb_status_message(st) : cudaGetErrorString(e));
      if (st) sb_status_free(st);
      cudaGetLastError();
      lf->graphs_off = true;
      return nullptr;
    }
    slot->direct_in = direct;
    graph_log(lf, "captured (" + std::to_string(slot->kernels) + " kernels)");
  }
  // refresh the staged inputs, then replay
  for (size_t i = 0; i < nin; ++i)
    if (lf->staged[i] && in[i]->bytes)
      SB_CUDA(cudaMemcpyAsync(lf->stage_buf[i], in[i]->ptr, in[i]->bytes, cudaMemcpyDeviceToDevice, stream));
  SB_CUDA(cudaGraphLaunch(slot->exec, stream));
  graph_log(lf, "replayed");
  // the replay launches the captured kernels
  launch_counter().fetch_add(slot->kernels, std::memory_order_relaxed);
  for (size_t j = 0; j < f.returns.size(); ++j) {
    auto* b = new sb_buffer();
    b->dev = s->dev;
    b->type = f.value_types[f.returns[j]];
    b->bytes = (size_t)b->type.numel() * dtype_bytes(b->type.dtype);
    b->ptr = outp[j];
    b->owned = false;
    b->slot = slot;
    out[j] = b;
  }
  slot->held.store((int)f.returns.size());
  *nout = f.returns.size();
  lf->calls++;
  *used = true;
  return nullptr;
}

sb_status* run_function(sb_session* s, LoadedFunction* lf, sb_buffer* const* in, size_t nin,
                        const int32_t* reduce, sb_buffer** out, size_t cap, size_t* nout) {
  const Function& f = *lf->plan.fn;
  if (nin != f.params.size())
    return make_status(SB_STATUS_INVALID_ARGUMENT, "@" + f.name + " expects " + std::to_string(f.params.size()) +
                                                       " inputs, got " + std::to_string(nin));
  for (size_t i = 0; i < nin; ++i) {
    if (!in[i]) return make_status(SB_STATUS_INVALID_ARGUMENT, "input " + std::to_string(i) + " is NULL");
    if (!(in[i]->type.shape == f.params[i].shape))
      return make_status(SB_STATUS_INVALID_ARGUMENT, "shape mismatch for input " + std::to_string(i) + ": got " +
                                                         in[i]->type.str() + ", expected " + f.params[i].str());
    if (in[i]->type.dtype != f.params[i].dtype)
      return make_status(SB_STATUS_INVALID_ARGUMENT, "element type mismatch for input " + std::to_string(i));
  }
  if (cap < f.returns.size())
    return make_status(SB_STATUS_INVALID_ARGUMENT, "output capacity " + std::to_string(cap) + " < " +
                                                       std::to_string(f.returns.size()));
  cudaStream_t stream = s->dev->stream;
  SB_CUDA(cudaSetDevice(s->dev->ordinal));
  const Plan& plan = lf->plan;
  // calls replay a CUDA graph from the second call on (run_graph)
  if (graphs_enabled() && !(s->opts.flags & SB_SESSION_FLAG_NO_CUDA_GRAPH) && !s->profiling && !lf->graphs_off) {
    bool used = false;
    sb_status* st = run_graph(s, lf, in, nin, reduce, out, nout, &used);
    if (st || used) return st;
  }
  // outputs
  std::vector<sb_buffer*> outs(f.returns.size(), nullptr);
  auto cleanup = [&]() {
    for (auto* b : outs) if (b) sb_buffer_release(b);
  };
  for (size_t j = 0; j < f.returns.size(); ++j) {
    sb_status* st = nullptr;
    outs[j] = new_device_buffer(s->dev, f.value_types[f.returns[j]], &st);
    if (!outs[j]) { cleanup(); return st; }
  }
  std::vector<void*> ptr(f.num_values(), nullptr);
  for (size_t i = 0; i < nin; ++i) ptr[i] = in[i]->ptr;
  for (auto& [v, p] : lf->const_ptr) ptr[v] = p;
  for (size_t j = 0; j < f.returns.size(); ++j)
    if (plan.output_step[j] >= 0) ptr[f.returns[j]] = outs[j]->ptr;
  for (int v : plan.materialized)
    if (!ptr[v] && plan.value_offset[v] >= 0) ptr[v] = (char*)lf->arena + plan.value_offset[v];

  // Data parallel, overlapped: each reduced output is all-reduced on the comm
  // stream once the step that writes it and every step that reads it have
  // been enqueued, in buckets of >= 8 MB (configurable), while later steps run
  // on `stream`.
  // Every rank has the same plan, so every rank issues the same buckets.
  const bool overlap = s->opts.world_size > 1 && reduce && s->dev->comm_stream;
  std::vector<std::vector<int>> ready_at(plan.steps.size());
  std::vector<int> bucket;
  size_t bucket_bytes = 0;
  // SHEAF_B200_ALLREDUCE_BUCKET_BYTES overrides the bucket size (tests use
  // small buckets to exercise many of them)
  size_t bucket_limit = 16u << 20;  // as in capture_reductions
  if (const char* bb = std::getenv("SHEAF_B200_ALLREDUCE_BUCKET_BYTES"))
    if (std::atoll(bb) > 0) bucket_limit = (size_t)std::atoll(bb);
  bool comm_used = false;
  if (overlap) {
    std::vector<int> last(f.num_values(), -1);
    for (int si = 0; si < (int)plan.steps.size(); ++si)
      for (int l : plan.steps[si].leaves) last[l] = si;
    std::vector<int> times(f.num_values(), 0);
    for (int v : f.returns) ++times[v];
    for (size_t j = 0; j < f.returns.size(); ++j) {
      if (reduce[j] == SB_REDUCE_NONE) continue;
      if (outs[j]->type.dtype != DType::F32) { cleanup(); return make_status(SB_STATUS_UNIMPLEMENTED, "reduce of non-f32 output"); }
      const int v = f.returns[j];
      // outputs copied after the steps, and values returned more than once
      // (their copies read the first buffer), go to the last bucket
      if (plan.output_step[j] < 0 || times[v] > 1) continue;
      ready_at[std::max(plan.output_step[j], last[v])].push_back((int)j);
    }
  }
  const std::function<sb_status*()>* red_flush = nullptr;  // deferred split-K reductions (during the steps)
  auto flush_bucket = [&]() -> sb_status* {
    if (bucket.empty()) return nullptr;
    if (red_flush)
      if (sb_status* st = (*red_flush)()) return st;
    const NcclApi& api = nccl_api();
    if (!s->nccl.comm) return make_status(SB_STATUS_FAILED_PRECONDITION, "NCCL communicator is not available");
    SB_CUDA(cudaEventRecord(s->dev->ready, stream));
    SB_CUDA(cudaStreamWaitEvent(s->dev->comm_stream, s->dev->ready, 0));
    api.group_start();
    for (int j : bucket) {
      ncclRedOp_t op = reduce[j] == SB_REDUCE_MEAN ? ncclAvg : ncclSum;
      ncclResult_t r = api.all_reduce(outs[j]->ptr, outs[j]->ptr, (size_t)outs[j]->type.numel(), ncclFloat32, op,
                                      s->nccl.comm, s->dev->comm_stream);
      if (r != ncclSuccess && r != ncclInProgress) {
        api.group_end();
        return make_status(SB_STATUS_INTERNAL, std::string("ncclAllReduce: ") + api.error_string(r));
      }
    }
    ncclResult_t r = api.group_end();
    if (r != ncclSuccess && r != ncclInProgress)
      return make_status(SB_STATUS_INTERNAL, std::string("ncclGroupEnd: ") + api.error_string(r));
    bucket.clear();
    bucket_bytes = 0;
    comm_used = true;
    return nccl_settle(s);
  };
  const BeforeStep before = [&](size_t si, const std::function<sb_status*()>& fl) -> sb_status* {
    red_flush = &fl;
    if (!overlap || si == 0) return nullptr;
    for (int j : ready_at[si - 1]) {
      bucket.push_back(j);
      bucket_bytes += outs[j]->bytes;
    }
    if (bucket_bytes >= bucket_limit) return flush_bucket();
    return nullptr;
  };
  {
    std::vector<void*> outp(outs.size());
    for (size_t j = 0; j < outs.size(); ++j) outp[j] = outs[j]->ptr;
    sb_status* e = enqueue_steps(s, lf, ptr, outp, before, false);
    red_flush = nullptr;
    if (e) { cleanup(); return e; }
  }
  // data-parallel combine of outputs
  if (overlap) {
    // the outputs of the last step and those copied above, then `stream`
    // waits for every bucket
    if (!plan.steps.empty())
      for (int j : ready_at.back()) bucket.push_back(j);
    std::vector<char> queued(f.returns.size(), 0);
    for (auto& r : ready_at)
      for (int j : r) queued[j] = 1;
    for (size_t j = 0; j < f.returns.size(); ++j)
      if (reduce[j] != SB_REDUCE_NONE && !queued[j]) bucket.push_back((int)j);
    if (sb_status* e = flush_bucket()) { cleanup(); return e; }
    if (comm_used) {
      SB_CUDA(cudaEventRecord(s->dev->reduced, s->dev->comm_stream));
      SB_CUDA(cudaStreamWaitEvent(stream, s->dev->reduced, 0));
    }
  } else if (s->opts.world_size > 1 && reduce) {
    if (!s->nccl.comm) { cleanup(); return make_status(SB_STATUS_FAILED_PRECONDITION, "NCCL communicator is not available"); }
    const NcclApi& api = nccl_api();
    api.group_start();
    for (size_t j = 0; j < f.returns.size(); ++j) {
      if (reduce[j] == SB_REDUCE_NONE) continue;
      if (outs[j]->type.dtype != DType::F32) { api.group_end(); cleanup(); return make_status(SB_STATUS_UNIMPLEMENTED, "reduce of non-f32 output"); }
      ncclRedOp_t op = reduce[j] == SB_REDUCE_MEAN ? ncclAvg : ncclSum;
      ncclResult_t r = api.all_reduce(outs[j]->ptr, outs[j]->ptr, (size_t)outs[j]->type.numel(), ncclFloat32, op,
                                      s->nccl.comm, stream);
      if (r != ncclSuccess && r != ncclInProgress) { api.group_end(); cleanup(); return make_status(SB_STATUS_INTERNAL, std::string("ncclAllReduce: ") + api.error_string(r)); }
    }
    ncclResult_t r = api.group_end();
    if (r != ncclSuccess && r != ncclInProgress) { cleanup(); return make_status(SB_STATUS_INTERNAL, std::string("ncclGroupEnd: ") + api.error_string(r)); }
    if (sb_status* e = nccl_settle(s)) { cleanup(); return e; }
  }
  SB_CUDA(cudaGetLastError());
  for (size_t j = 0; j < f.returns.size(); ++j) out[j] = outs[j];
  *nout = f.returns.size();
  lf->calls++;
  return nullptr;
}

}  // namespace
}  // namespace sb

using namespace sb;

extern "C" {

sb_status_code sb_status_code_of(const sb_status* s) { return s ? s->code : SB_STATUS_OK; }
const char* sb_status_message(const sb_status* s) { return s ? s->message.c_str() : "OK"; }
void sb_status_free(sb_status* s) { delete s; }
const char* sb_version(void) { return "sheaf_b200 0.1 (sm_100a)"; }

uint64_t sb_kernel_launch_count(void) { return sb::launch_counter().load(std::memory_order_relaxed); }

void sb_session_options_initialize(sb_session_options* o) {
  std::memset(o, 0, sizeof *o);
  o->device_ordinal = 0;
  o->precision = SB_PRECISION_TF32;
  o->rank = 0;
  o->world_size = 1;
  o->collective_timeout_ms = 600000;
}

sb_status* sb_session_create(const sb_session_options* o, sb_session** out) {
  if (!o || !out) return make_status(SB_STATUS_INVALID_ARGUMENT, "NULL argument");
  *out = nullptr;
  if (o->precision < 0 || o->precision > 2) return make_status(SB_STATUS_INVALID_ARGUMENT, "bad precision");
  if (o->world_size < 1 || o->rank < 0 || o->rank >= o->world_size)
    return make_status(SB_STATUS_INVALID_ARGUMENT, "bad rank / world_size");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) {
    cudaGetLastError();
    return make_status(SB_STATUS_UNAVAILABLE, "no CUDA device is available");
  }
  if (o->device_ordinal < 0 || o->device_ordinal >= n)
    return make_status(SB_STATUS_INVALID_ARGUMENT, "device ordinal out of range");
  cudaDeviceProp prop;
  SB_CUDA(cudaGetDeviceProperties(&prop, o->device_ordinal));
  if (prop.major != 10)
    return make_status(SB_STATUS_UNAVAILABLE, std::string("device ") + prop.name +
                                                  " is not an sm_100 (B200-class) GPU; this library is built for sm_100a only");
  auto s = std::make_unique<sb_session>();
  s->opts = *o;
  s->cache_dir = o->kernel_cache_dir ? o->kernel_cache_dir : default_cache_dir();
  s->dev = std::make_shared<Device>();
  s->dev->ordinal = o->device_ordinal;
  SB_CUDA(cudaSetDevice(o->device_ordinal));
  SB_CUDA(cudaStreamCreateWithFlags(&s->dev->stream, cudaStreamNonBlocking));
  if (o->world_size > 1 && (o->flags & SB_SESSION_FLAG_OVERLAP_ALLREDUCE)) {
    SB_CUDA(cudaStreamCreateWithFlags(&s->dev->comm_stream, cudaStreamNonBlocking));
    SB_CUDA(cudaEventCreateWithFlags(&s->dev->ready, cudaEventDisableTiming));
    SB_CUDA(cudaEventCreateWithFlags(&s->dev->reduced, cudaEventDisableTiming));
  }
  if (o->world_size > 1) {
    const NcclApi& api = nccl_api();
    if (!api.ok) return make_status(SB_STATUS_UNAVAILABLE, api.error);
    ncclUniqueId id;
    std::memcpy(&id, o->nccl_unique_id, sizeof id);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclComm_t comm = nullptr;
    ncclResult_t r = api.init_rank_config(&comm, o->world_size, id, o->rank, &cfg);
    auto t0 = std::chrono::steady_clock::now();
    int64_t tmo = o->collective_timeout_ms > 0 ? o->collective_timeout_ms : 600000;
    while (r == ncclInProgress || r == ncclSuccess) {
      ncclResult_t ae = ncclInProgress;
      if (comm) api.async_error(comm, &ae);
      if (ae == ncclSuccess) break;
      if (ae != ncclInProgress) { r = ae; break; }
      if (std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count() > tmo) {
        if (comm) api.comm_abort(comm);
        return make_status(SB_STATUS_DEADLINE_EXCEEDED, "NCCL communicator initialization timed out");
      }
      std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
    if (r != ncclSuccess && r != ncclInProgress) {
      if (comm) api.comm_abort(comm);
      return make_status(SB_STATUS_UNAVAILABLE, std::string("ncclCommInitRankConfig: ") + api.error_string(r));
    }
    s->nccl.comm = comm;
  }
  *out = s.release();
  return nullptr;
}

void sb_session_release(sb_session* s) {
  if (!s) return;
  cudaSetDevice(s->dev->ordinal);
  cudaStreamSynchronize(s->dev->stream);
  // graphs that hold NCCL operations go before the communicator (the slots
  // themselves may outlive the session while the caller holds outputs)
  for (auto& m : s->modules)
    for (auto& lf : m->fns)
      for (auto& sl : lf->slots)
        if (sl->exec) {
          cudaGraphExecDestroy(sl->exec);
          sl->exec = nullptr;
        }
  if (s->nccl.comm) nccl_api().comm_destroy(s->nccl.comm);
  for (auto& m : s->modules) {
    for (auto& lf : m->fns) {
      for (auto& [v, p] : lf->const_ptr) cudaFree(p);
      if (lf->arena) cudaFree(lf->arena);
      if (lf->ws) cudaFree(lf->ws);
      for (void* p : lf->stage_buf)
        if (p) cudaFree(p);
    }
    for (auto lib : m->libs) cudaLibraryUnload(lib);
  }
  delete s;
}

sb_status* sb_session_synchronize(sb_session* s) {
  if (!s) return make_status(SB_STATUS_INVALID_ARGUMENT, "NULL session");
  std::lock_guard<std::mutex> g(s->mu);
  return wait_stream(s, s->opts.world_size > 1 ? deadline_ms(s) : 0);
}

sb_status* sb_session_allocator_stats(sb_session* s, sb_allocator_stats* o) {
  if (!s || !o) return make_status(SB_STATUS_INVALID_ARGUMENT, "NULL argument");
  std::memset(o, 0, sizeof *o);
  o->device_bytes_peak = s->dev->peak;
  o->device_bytes_allocated = s->dev->allocated;
  o->device_bytes_freed = s->dev->freed;
  return nullptr;
}

void* sb_session_cuda_stream(sb_session* s) { return s ? (void*)s->dev->stream : nullptr; }

sb_status* sb_session_set_profiling(sb_session* s, int enable) {
  if (!s) return make_status(SB_STATUS_INVALID_ARGUMENT, "NULL session");
  std::lock_guard<std::mutex> g(s->mu);
  s->profiling = enable != 0;
  return nullptr;
}

sb_status* sb_session_profile_report(sb_session* s, int reset, char* out, size_t cap, size_t* out_len) {
  if (!s) return make_status(SB_STATUS_INVALID_ARGUMENT, "NULL session");
  std::lock_guard<std::mutex> g(s->mu);
  SB_CUDA(cudaSetDevice(s->dev->ordinal));
  SB_CUDA(cudaStreamSynchronize(s->dev->stream));
  for (auto& p : s->pending) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, p.a, p.b);
    auto* lf = p.fn;
    if (lf->prof_ms.size() != lf->plan.steps.size()) {
      lf->prof_ms.assign(lf->plan.steps.size(), 0.0);
      lf->prof_n.assign(lf->plan.steps.size(), 0);
      lf->prof_launches.assign(lf->plan.steps.size(), 0);
    }
    lf->prof_ms[p.step] += ms;
    lf->prof_n[p.step] += 1;
    lf->prof_launches[p.step] = p.launches;
    s->free_events.push_back(p.a);
    s->free_events.push_back(p.b);
  }
  s->pending.clear();
  std::ostringstream os;
  os.precision(9);
  os << "function,step,kind,kernel,calls,total_ms,elements,bytes,flops,launches_per_call\n";
  static const char* kinds[] = {"loop", "reduce", "gemm", "attention", "sort", "convert", "scatter"};
  for (auto& m : s->modules)
    for (auto& lf : m->fns) {
      if (lf->prof_ms.empty()) continue;
      for (size_t i = 0; i < lf->plan.steps.size(); ++i) {
        const Step& st = lf->plan.steps[i];
        if (!lf->prof_n[i]) continue;
        os << lf->qname << "," << i << "," << kinds[(int)st.kind] << ","
           << step_name(st) << "," << lf->prof_n[i] << "," << lf->prof_ms[i]
           << "," << st.elements << "," << st.bytes_moved << "," << st.flops << "," << lf->prof_launches[i]
           << "\n";
      }
      if (reset) {
        std::fill(lf->prof_ms.begin(), lf->prof_ms.end(), 0.0);
        std::fill(lf->prof_n.begin(), lf->prof_n.end(), 0);
      }
    }
  std::string r = os.str();
  if (out_len) *out_len = r.size();
  if (out && cap) {
    size_t n = std::min(cap - 1, r.size());
    std::memcpy(out, r.data(), n);
    out[n] = 0;
  }
  return nullptr;
}

// Ahead-of-time bundle: "SB200BND", u32 version 1, i32 precision, u32 flags,
// u64 text length + StableHLO text, u32 chunk count, then per chunk a
// 32-character key, u64 size and the cubin.  Little-endian.
extern "C++" {
namespace sb {
namespace {
constexpr char kBundleMagic[8] = {'S', 'B', '2', '0', '0', 'B', 'N', 'D'};
template <typename T>
void put(std::string& o, T v) {
  o.append((const char*)&v, sizeof v);
}
template <typename T>
bool get(const uint8_t*& p, const uint8_t* e, T* v) {
  if ((size_t)(e - p) < sizeof(T)) return false;
  std::memcpy(v, p, sizeof(T));
  p += sizeof(T);
  return true;
}
}  // namespace
}  // namespace sb
}

sb_status* sb_module_build_bundle(const char* text, size_t len, int32_t precision, uint32_t flags, uint8_t* out,
                                  size_t cap, size_t* out_len) {
  using namespace sb;
  if (!text || !out_len) return make_status(SB_STATUS_INVALID_ARGUMENT, "NULL argument");
  if (precision < 0 || precision > 2) return make_status(SB_STATUS_INVALID_ARGUMENT, "unknown precision");
  std::string err;
  const std::string src(text, len);
  auto mod = parse_module(src, &err);
  if (!mod) return make_status(SB_STATUS_INVALID_ARGUMENT, err);
  std::vector<CubinChunk> all;
  for (auto& f : mod->funcs) {
    Plan p;
    try {
      p = build_plan(f, (Precision)precision, !(flags & SB_SESSION_FLAG_NO_ATTENTION_FUSION));
    } catch (const std::exception& e) {
      return make_status(SB_STATUS_UNIMPLEMENTED, "planning @" + f.name + ": " + e.what());
    }
    std::vector<CubinChunk> chunks = split_source(p.snippets, p.prelude, 16);
    try {
      if (!p.snippets.empty()) compile_chunks(chunks, default_cache_dir());
    } catch (const std::exception& e) {
      return make_status(SB_STATUS_INTERNAL, "kernel compilation for @" + f.name + " failed: " + e.what());
    }
    if (!p.snippets.empty())
      for (auto& c : chunks) all.push_back(std::move(c));
  }
  std::string o(kBundleMagic, 8);
  put<uint32_t>(o, 1);
  put<int32_t>(o, precision);
  put<uint32_t>(o, flags);
  put<uint64_t>(o, src.size());
  o += src;
  put<uint32_t>(o, (uint32_t)all.size());
  for (auto& c : all) {
    const std::string key = chunk_key(c.source);
    o += key;
    put<uint64_t>(o, c.cubin.size());
    o.append((const char*)c.cubin.data(), c.cubin.size());
  }
  *out_len = o.size();
  if (!out) return nullptr;
  if (cap < o.size()) return make_status(SB_STATUS_RESOURCE_EXHAUSTED, "bundle buffer too small");
  std::memcpy(out, o.data(), o.size());
  return nullptr;
}

sb_status* sb_session_load_bundle(sb_session* s, const uint8_t* data, size_t len) {
  using namespace sb;
  if (!s || !data) return make_status(SB_STATUS_INVALID_ARGUMENT, "NULL argument");
  const uint8_t *p = data, *e = data + len;
  auto bad = [](const char* what) { return make_status(SB_STATUS_INVALID_ARGUMENT, std::string("bundle: ") + what); };
  if (len < 8 || std::memcmp(p, kBundleMagic, 8) != 0) return bad("not a sheaf_b200 bundle");
  p += 8;
  uint32_t version = 0, flags = 0, n = 0;
  int32_t precision = 0;
  uint64_t tlen = 0;
  if (!get(p, e, &version) || version != 1) return bad("unsupported version");
  if (!get(p, e, &precision) || !get(p, e, &flags) || !get(p, e, &tlen) || (uint64_t)(e - p) < tlen)
    return bad("truncated header");
  if (precision != s->opts.precision) return bad("built for another precision than this session's");
  if ((flags & SB_SESSION_FLAG_NO_ATTENTION_FUSION) != (s->opts.flags & SB_SESSION_FLAG_NO_ATTENTION_FUSION))
    return bad("built with other planning flags than this session's");
  std::string text((const char*)p, (size_t)tlen);
  p += tlen;
  if (!get(p, e, &n)) return bad("truncated chunk table");
  Prebuilt pre;
  for (uint32_t i = 0; i < n; ++i) {
    uint64_t sz = 0;
    if ((size_t)(e - p) < 32) return bad("truncated chunk key");
    std::string key((const char*)p, 32);
    p += 32;
    if (!get(p, e, &sz) || (uint64_t)(e - p) < sz) return bad("truncated cubin");
    pre[key].assign(p, p + sz);
    p += sz;
  }
  std::lock_guard<std::mutex> g(s->mu);
  return load_module(s, text, &pre);
}

sb_status* sb_session_load_stablehlo(sb_session* s, const char* text, size_t len) {
  if (!s || !text) return make_status(SB_STATUS_INVALID_ARGUMENT, "NULL argument");
  std::lock_guard<std::mutex> g(s->mu);
  return load_module(s, std::string(text, len));
}

int sb_session_has_function(sb_session* s, const char* name) {
  if (!s || !name) return 0;
  std::lock_guard<std::mutex> g(s->mu);
  return s->by_name.count(name) ? 1 : 0;
}

sb_status* sb_session_call(sb_session* s, const char* name, sb_buffer* const* inputs, size_t n_in,
                           const int32_t* reduce, sb_buffer** outputs, size_t cap, size_t* n_out) {
  if (!s || !name || (n_in && !inputs) || !n_out) return make_status(SB_STATUS_INVALID_ARGUMENT, "NULL argument");
  *n_out = 0;
  std::lock_guard<std::mutex> g(s->mu);
  if (s->nccl.aborted) return make_status(SB_STATUS_FAILED_PRECONDITION, "NCCL communicator was aborted");
  auto it = s->by_name.find(name);
  if (it == s->by_name.end()) return make_status(SB_STATUS_NOT_FOUND, std::string("function not found: ") + name);
  return run_function(s, it->second, inputs, n_in, reduce, outputs, cap, n_out);
}

sb_status* sb_buffer_allocate_copy(sb_session* s, size_t rank, const uint64_t* shape, uint32_t et,
                                   const void* host, size_t bytes, sb_buffer** out) {
  if (!s || !out || (rank && !shape)) return make_status(SB_STATUS_INVALID_ARGUMENT, "NULL argument");
  Type t;
  if (!etype_to_dtype(et, &t.dtype)) return make_status(SB_STATUS_INVALID_ARGUMENT, "unsupported element type");
  for (size_t i = 0; i < rank; ++i) t.shape.push_back((int64_t)shape[i]);
  size_t need = (size_t)t.numel() * dtype_bytes(t.dtype);
  if (bytes != need)
    return make_status(SB_STATUS_INVALID_ARGUMENT, "byte length " + std::to_string(bytes) + " does not match shape (" +
                                                       std::to_string(need) + ")");
  if (need && !host) return make_status(SB_STATUS_INVALID_ARGUMENT, "NULL host data");
  std::lock_guard<std::mutex> g(s->mu);
  SB_CUDA(cudaSetDevice(s->dev->ordinal));
  sb_status* st = nullptr;
  sb_buffer* b = new_device_buffer(s->dev, t, &st);
  if (!b) return st;
  if (need) {
    cudaError_t e = cudaMemcpyAsync(b->ptr, host, need, cudaMemcpyHostToDevice, s->dev->stream);
    if (e != cudaSuccess) {
      sb_buffer_release(b);
      return cuda_status(e, "cudaMemcpyAsync(H2D)");
    }
  }
  *out = b;
  return nullptr;
}

sb_status* sb_buffer_wrap_device(sb_session* s, size_t rank, const uint64_t* shape, uint32_t et, void* dptr,
                                 size_t bytes, sb_buffer** out) {
  if (!s || !out || (rank && !shape)) return make_status(SB_STATUS_INVALID_ARGUMENT, "NULL argument");
  Type t;
  if (!etype_to_dtype(et, &t.dtype)) return make_status(SB_STATUS_INVALID_ARGUMENT, "unsupported element type");
  for (size_t i = 0; i < rank; ++i) t.shape.push_back((int64_t)shape[i]);
  if (bytes != (size_t)t.numel() * dtype_bytes(t.dtype))
    return make_status(SB_STATUS_INVALID_ARGUMENT, "byte length does not match shape");
  if (((uintptr_t)dptr) & 15)
    return make_status(SB_STATUS_INVALID_ARGUMENT, "device pointer must be 16-byte aligned");
  auto* b = new sb_buffer();
  b->type = t;
  b->bytes = bytes;
  b->ptr = dptr;
  b->owned = false;
  *out = b;
  return nullptr;
}

void sb_adamw_options_initialize(sb_adamw_options* o) {
  if (!o) return;
  o->learning_rate = 1e-3f;
  o->beta1 = 0.9f;
  o->beta2 = 0.999f;
  o->epsilon = 1e-8f;
  o->weight_decay = 0.f;
  o->max_grad_norm = 0.f;
  o->step = 0;
}

sb_status* sb_optimizer_adamw_step(sb_session* s, size_t n, sb_buffer* const* params, sb_buffer* const* grads,
                                   sb_buffer* const* m, sb_buffer* const* v, const sb_adamw_options* o,
                                   float* out_global_norm) {
  using namespace sb;
  if (!s || !o || (n && (!params || !grads || !m || !v)))
    return make_status(SB_STATUS_INVALID_ARGUMENT, "NULL argument");
  if (n > (size_t)INT32_MAX) return make_status(SB_STATUS_INVALID_ARGUMENT, "too many leaves");
  if (o->step < 0) return make_status(SB_STATUS_INVALID_ARGUMENT, "negative step");
  // fixed partition of every leaf into chunks of at most 16384 elements
  constexpr int64_t kChunk = 16384;
  std::vector<OptLeaf> leaves(n);
  std::vector<OptChunk> chunks;
  for (size_t i = 0; i < n; ++i) {
    sb_buffer* bs[4] = {params[i], grads[i], m[i], v[i]};
    for (int k = 0; k < 4; ++k) {
      if (!bs[k]) return make_status(SB_STATUS_INVALID_ARGUMENT, "NULL buffer in leaf " + std::to_string(i));
      if (bs[k]->type.dtype != DType::F32)
        return make_status(SB_STATUS_INVALID_ARGUMENT, "leaf " + std::to_string(i) + ": buffers must be f32");
      if (bs[k]->dev.get() != s->dev.get())
        return make_status(SB_STATUS_INVALID_ARGUMENT, "leaf " + std::to_string(i) + ": buffer of another session");
      if (bs[k]->bytes != params[i]->bytes)
        return make_status(SB_STATUS_INVALID_ARGUMENT,
                           "leaf " + std::to_string(i) + ": parameter, gradient and moment sizes differ");
    }
    const int64_t count = (int64_t)(params[i]->bytes / 4);
    leaves[i] = OptLeaf{(float*)params[i]->ptr, (const float*)grads[i]->ptr, (float*)m[i]->ptr, (float*)v[i]->ptr,
                        count};
    for (int64_t off = 0; off < count; off += kChunk)
      chunks.push_back(OptChunk{(int)i, off, std::min(kChunk, count - off)});
  }
  if (chunks.size() > (size_t)INT32_MAX) return make_status(SB_STATUS_INVALID_ARGUMENT, "too many elements");
  std::lock_guard<std::mutex> g(s->mu);
  SB_CUDA(cudaSetDevice(s->dev->ordinal));
  if (chunks.empty()) {
    if (out_global_norm) *out_global_norm = 0.f;
    return nullptr;
  }
  // scalar terms in double, as Sheaf evaluates scalars before they meet tensors
  const double t1 = (double)o->step + 1.0;
  AdamwScalars a;
  a.lr = o->learning_rate;
  a.b1 = o->beta1;
  a.b2 = o->beta2;
  a.one_minus_b1 = (float)(1.0 - (double)o->beta1);
  a.one_minus_b2 = (float)(1.0 - (double)o->beta2);
  a.eps = o->epsilon;
  a.wd = o->weight_decay;
  a.bc_m = (float)(1.0 / (1.0 - std::pow((double)o->beta1, t1)));
  a.bc_v = (float)(1.0 / (1.0 - std::pow((double)o->beta2, t1)));
  a.max_norm = o->max_grad_norm;
  a.clip = o->max_grad_norm > 0.f ? 1 : 0;
  const size_t lb = n * sizeof(OptLeaf), cb = chunks.size() * sizeof(OptChunk);
  const size_t pb = chunks.size() * sizeof(float);
  const size_t off_c = (lb + 255) & ~(size_t)255, off_p = (off_c + cb + 255) & ~(size_t)255;
  const size_t off_n = (off_p + pb + 255) & ~(size_t)255, total = off_n + 256;
  void* ws = nullptr;
  SB_CUDA(cudaMallocAsync(&ws, total, s->dev->stream));
  char* base = (char*)ws;
  // pageable sources: the copies are staged before cudaMemcpyAsync returns
  cudaError_t e = cudaMemcpyAsync(base, leaves.data(), lb, cudaMemcpyHostToDevice, s->dev->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(base + off_c, chunks.data(), cb, cudaMemcpyHostToDevice, s->dev->stream);
  if (e == cudaSuccess)
    e = adamw_step((const OptLeaf*)base, (const OptChunk*)(base + off_c), (int)chunks.size(), (float*)(base + off_p),
                   out_global_norm ? (float*)(base + off_n) : nullptr, a, s->dev->stream);
  if (e == cudaSuccess && out_global_norm)
    e = cudaMemcpyAsync(out_global_norm, base + off_n, sizeof(float), cudaMemcpyDeviceToHost, s->dev->stream);
  cudaFreeAsync(ws, s->dev->stream);
  if (e != cudaSuccess) return cuda_status(e, "sb_optimizer_adamw_step");
  if (out_global_norm) return wait_stream(s, s->opts.world_size > 1 ? deadline_ms(s) : 0);
  return nullptr;
}

sb_status* sb_buffer_d2h(sb_session* s, sb_buffer* b, void* host, size_t bytes, int64_t timeout_ms) {
  if (!s || !b || (bytes && !host)) return make_status(SB_STATUS_INVALID_ARGUMENT, "NULL argument");
  if (bytes != b->bytes) return make_status(SB_STATUS_INVALID_ARGUMENT, "byte length does not match buffer");
  std::lock_guard<std::mutex> g(s->mu);
  SB_CUDA(cudaSetDevice(s->dev->ordinal));
  if (bytes) SB_CUDA(cudaMemcpyAsync(host, b->ptr, bytes, cudaMemcpyDeviceToHost, s->dev->stream));
  int64_t tmo = timeout_ms;
  if (s->opts.world_size > 1 && tmo <= 0) tmo = deadline_ms(s);
  return wait_stream(s, tmo);
}

void sb_buffer_retain(sb_buffer* b) {
  if (b) b->refs.fetch_add(1);
}

void sb_buffer_release(sb_buffer* b) {
  if (!b) return;
  if (b->refs.fetch_sub(1) != 1) return;
  if (b->slot) {
    b->slot->held.fetch_sub(1);
    delete b;
    return;
  }
  if (b->owned && b->ptr && b->dev) {
    cudaSetDevice(b->dev->ordinal);
    cudaFreeAsync(b->ptr, b->dev->stream);
    b->dev->note_free(b->bytes);
  }
  delete b;
}

size_t sb_buffer_rank(const sb_buffer* b) { return b ? b->type.shape.size() : 0; }
uint64_t sb_buffer_dim(const sb_buffer* b, size_t i) {
  return (b && i < b->type.shape.size()) ? (uint64_t)b->type.shape[i] : 0;
}
uint32_t sb_buffer_element_type(const sb_buffer* b) { return b ? dtype_to_etype(b->type.dtype) : 0; }
size_t sb_buffer_byte_length(const sb_buffer* b) { return b ? b->bytes : 0; }
void* sb_buffer_device_pointer(const sb_buffer* b) { return b ? b->ptr : nullptr; }

sb_status* sb_nccl_get_unique_id(uint8_t out[128]) {
  if (!out) return make_status(SB_STATUS_INVALID_ARGUMENT, "NULL argument");
  const NcclApi& api = nccl_api();
  if (!api.ok) return make_status(SB_STATUS_UNAVAILABLE, api.error);
  ncclUniqueId id;
  ncclResult_t r = api.get_unique_id(&id);
  if (r != ncclSuccess) return make_status(SB_STATUS_UNAVAILABLE, std::string("ncclGetUniqueId: ") + api.error_string(r));
  std::memcpy(out, &id, 128);
  return nullptr;
}

sb_status* sb_module_inspect(const char* text, size_t len, int32_t precision, char* report, size_t cap) {
  if (!text) return make_status(SB_STATUS_INVALID_ARGUMENT, "NULL argument");
  std::string err;
  auto mod = parse_module(std::string(text, len), &err);
  if (!mod) return make_status(SB_STATUS_INVALID_ARGUMENT, err);
  std::ostringstream os;
  for (auto& f : mod->funcs) {
    Plan p;
    try {
      p = build_plan(f, (Precision)precision);
    } catch (const std::exception& e) {
      return make_status(SB_STATUS_UNIMPLEMENTED, "planning @" + f.name + ": " + e.what());
    }
    std::vector<CubinChunk> chunks = split_source(p.snippets, p.prelude, 16);
    try {
      if (!p.snippets.empty()) compile_chunks(chunks, default_cache_dir());
    } catch (const std::exception& e) {
      return make_status(SB_STATUS_INTERNAL, "kernel compilation for @" + f.name + " failed: " + e.what());
    }
    size_t cubin = 0;
    for (auto& c : chunks) cubin += c.cubin.size();
    os << f.name << ": ops=" << f.ops.size() << " " << p.summary() << " cubin_bytes=" << cubin << "\n";
  }
  std::string r = os.str();
  if (report && cap) {
    size_t n = std::min(cap - 1, r.size());
    std::memcpy(report, r.data(), n);
    report[n] = 0;
  }
  return nullptr;
}

sb_status* sb_module_plan_steps(const char* text, size_t len, const char* fn, int32_t precision, char* out,
                                 size_t cap, size_t* out_len) {
  if (!text || !fn) return make_status(SB_STATUS_INVALID_ARGUMENT, "NULL argument");
  std::string err;
  auto mod = parse_module(std::string(text, len), &err);
  if (!mod) return make_status(SB_STATUS_INVALID_ARGUMENT, err);
  const Function* f = mod->find(fn);
  if (!f) return make_status(SB_STATUS_NOT_FOUND, std::string("function not found: ") + fn);
  Plan p;
  try {
    p = build_plan(*f, (Precision)precision);
  } catch (const std::exception& e) {
    return make_status(SB_STATUS_UNIMPLEMENTED, e.what());
  }
  std::ostringstream os;
  os.precision(17);
  os << "step,kind,kernel,elements,bytes,flops,batch,M,N,K,sab,sam,sak,sbb,sbk,sbn,epi,deferred_sums,root_offset\n";
  static const char* kinds[] = {"loop", "reduce", "gemm", "attention", "sort", "convert", "scatter"};
  for (size_t i = 0; i < p.steps.size(); ++i) {
    const Step& st = p.steps[i];
    const GemmDesc& g = st.gemm;
    os << i << "," << kinds[(int)st.kind] << "," << step_name(st) << ","
       << st.elements << "," << st.bytes_moved << "," << st.flops << "," << g.batch << "," << g.M << "," << g.N
       << "," << g.K << "," << g.sab << "," << g.sam << "," << g.sak << "," << g.sbb << "," << g.sbk << ","
       << g.sbn << "," << g.epi << "," << (st.finish_deferred ? st.col_finish.size() : 0) << ","
       << (st.kind == StepKind::Convert ? p.shadows[st.shadow].offset : p.value_offset[st.root]) << "\n";
  }
  std::string r = os.str();
  if (out_len) *out_len = r.size();
  if (out && cap) {
    size_t n = std::min(cap - 1, r.size());
    std::memcpy(out, r.data(), n);
    out[n] = 0;
  }
  return nullptr;
}

sb_status* sb_module_kernel_source(const char* text, size_t len, const char* fn, char* out, size_t cap,
                                   size_t* out_len) {
  if (!text || !fn) return make_status(SB_STATUS_INVALID_ARGUMENT, "NULL argument");
  std::string err;
  auto mod = parse_module(std::string(text, len), &err);
  if (!mod) return make_status(SB_STATUS_INVALID_ARGUMENT, err);
  const Function* f = mod->find(fn);
  if (!f) return make_status(SB_STATUS_NOT_FOUND, std::string("function not found: ") + fn);
  Plan p;
  try {
    p = build_plan(*f, Precision::TF32);
  } catch (const std::exception& e) {
    return make_status(SB_STATUS_UNIMPLEMENTED, e.what());
  }
  if (out_len) *out_len = p.source.size();
  if (out && cap) {
    size_t n = std::min(cap - 1, p.source.size());
    std::memcpy(out, p.source.data(), n);
    out[n] = 0;
  }
  return nullptr;
}

}  // extern "C"
