// runtime.cpp -- the C ABI of include/topos_b200.h: lazy device set-up and
// poisoning, NVRTC compilation of the emitted kernels, device buffers (one
// liveness-planned arena per plan), the CUDA-graph replay of a plan, device
// parameters, optimizer steps and the NCCL gradient exchange.
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <nvrtc.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <sstream>
#include <stdexcept>
#include <string>
#include <set>
#include <vector>

#include "engine.h"
#include "kernels.h"
#include "launch.h"

namespace {

thread_local std::string g_error;
std::mutex g_mutex;
int g_state = -1;  // -1 unknown, else TB_* status
std::string g_status_message;

struct Failure : std::runtime_error {
  int code;
  Failure(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] void runtime_fail(const std::string& m) { throw Failure(TB_RUNTIME, m); }

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) runtime_fail(std::string(what) + ": " + cudaGetErrorString(e));
}
// Driver entry points, resolved through the runtime so that the library does
// not link libcuda (it loads on machines without a driver and reports
// PlatformUnsupported there).
struct Driver {
  CUresult (*GetErrorString)(CUresult, const char**) = nullptr;
  CUresult (*ModuleLoadData)(CUmodule*, const void*) = nullptr;
  CUresult (*ModuleGetFunction)(CUfunction*, CUmodule, const char*) = nullptr;
  CUresult (*LaunchKernelEx)(const CUlaunchConfig*, CUfunction, void**, void**) = nullptr;
  CUresult (*FuncSetAttribute)(CUfunction, CUfunction_attribute, int) = nullptr;
};
Driver g_driver;

}  // namespace

bool tb::pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("TB_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

namespace {

bool load_driver() {
  auto get = [](const char* name, void** fn) {
    cudaDriverEntryPointQueryResult q;
    return cudaGetDriverEntryPoint(name, fn, cudaEnableDefault, &q) == cudaSuccess &&
           q == cudaDriverEntryPointSuccess && *fn;
  };
  return get("cuGetErrorString", (void**)&g_driver.GetErrorString) &&
         get("cuModuleLoadData", (void**)&g_driver.ModuleLoadData) &&
         get("cuModuleGetFunction", (void**)&g_driver.ModuleGetFunction) &&
         get("cuLaunchKernelEx", (void**)&g_driver.LaunchKernelEx) &&
         get("cuFuncSetAttribute", (void**)&g_driver.FuncSetAttribute);
}

void check(CUresult e, const char* what) {
  if (e != CUDA_SUCCESS) {
    const char* s = nullptr;
    if (g_driver.GetErrorString) g_driver.GetErrorString(e, &s);
    runtime_fail(std::string(what) + ": " + (s ? s : std::to_string((int)e)));
  }
}

// Lazy set-up, once per process (backend/cuda/kernels/mod.rs:36-58): a device
// must exist; everything else is per plan.
int ensure_ready() {
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_state >= 0) return g_state;
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0) {
    g_state = TB_PLATFORM_UNSUPPORTED;
    g_status_message = e != cudaSuccess ? cudaGetErrorString(e) : "no CUDA device";
    return g_state;
  }
  if (cudaFree(nullptr) != cudaSuccess || !load_driver()) {
    g_state = TB_INITIALIZATION;
    g_status_message = "CUDA context or driver entry points unavailable";
    return g_state;
  }
  g_state = TB_OK;
  return g_state;
}

void poison(const std::string& why) {
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_state == TB_OK) {
    g_state = TB_POISONED;
    g_status_message = why;
  }
}

template <class F>
int guarded(F&& body, bool needs_device = true) {
  try {
    if (needs_device) {
      int s = ensure_ready();
      if (s != TB_OK) {
        g_error = "backend unavailable: " + g_status_message;
        return s;
      }
    }
    return body();
  } catch (const Failure& f) {
    g_error = f.what();
    if (f.code == TB_RUNTIME) poison(f.what());
    return f.code;
  } catch (const std::exception& e) {
    g_error = e.what();
    return TB_INVALID;
  }
}

// ---- NVRTC: one program per distinct source text, cached for the process
struct CompiledModule {
  CUmodule module = nullptr;
  int device = -1;
};
std::map<std::pair<std::string, int>, CompiledModule> g_modules;
std::mutex g_module_mutex;

CUmodule compile_module(const std::string& source, int device) {
  std::lock_guard<std::mutex> lock(g_module_mutex);
  auto key = std::make_pair(source, device);
  auto it = g_modules.find(key);
  if (it != g_modules.end()) return it->second.module;
  nvrtcProgram prog;
  if (nvrtcCreateProgram(&prog, source.c_str(), "topos_b200_fused.cu", 0, nullptr, nullptr) !=
      NVRTC_SUCCESS)
    runtime_fail("nvrtcCreateProgram failed");
  const char* opts[] = {"-arch=sm_100a", "--fmad=false", "-prec-div=true", "-prec-sqrt=true",
                        "-ftz=false", "-std=c++17", "-default-device", "-lineinfo"};
  nvrtcResult r = nvrtcCompileProgram(prog, sizeof(opts) / sizeof(opts[0]), opts);
  if (r != NVRTC_SUCCESS) {
    size_t n = 0;
    nvrtcGetProgramLogSize(prog, &n);
    std::string log(n, '\0');
    nvrtcGetProgramLog(prog, &log[0]);
    nvrtcDestroyProgram(&prog);
    throw Failure(TB_INVALID, "NVRTC compile failed:\n" + log.substr(0, 4000));
  }
  size_t size = 0;
  nvrtcGetCUBINSize(prog, &size);
  std::string cubin(size, '\0');
  nvrtcGetCUBIN(prog, &cubin[0]);
  nvrtcDestroyProgram(&prog);
  CUmodule mod;
  check(g_driver.ModuleLoadData(&mod, cubin.data()), "cuModuleLoadData");
  g_modules[key] = CompiledModule{mod, device};
  return mod;
}

// ---- NCCL, loaded at run time (the process may already hold torch's copy)
struct Nccl {
  void* handle = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};
Nccl* nccl() {
  static Nccl n;
  static bool tried = false;
  if (tried) return n.handle ? &n : nullptr;
  tried = true;
  const char* names[] = {"libnccl.so.2", "libnccl.so"};
  for (const char* name : names) {
    n.handle = dlopen(name, RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (!n.handle) n.handle = dlopen(name, RTLD_NOW | RTLD_GLOBAL);
    if (n.handle) break;
  }
  if (!n.handle) return nullptr;
  n.GetUniqueId = (decltype(n.GetUniqueId))dlsym(n.handle, "ncclGetUniqueId");
  n.CommInitRank = (decltype(n.CommInitRank))dlsym(n.handle, "ncclCommInitRank");
  n.CommDestroy = (decltype(n.CommDestroy))dlsym(n.handle, "ncclCommDestroy");
  n.CommAbort = (decltype(n.CommAbort))dlsym(n.handle, "ncclCommAbort");
  n.AllReduce = (decltype(n.AllReduce))dlsym(n.handle, "ncclAllReduce");
  n.AllGather = (decltype(n.AllGather))dlsym(n.handle, "ncclAllGather");
  n.GroupStart = (decltype(n.GroupStart))dlsym(n.handle, "ncclGroupStart");
  n.GroupEnd = (decltype(n.GroupEnd))dlsym(n.handle, "ncclGroupEnd");
  n.GetErrorString = (decltype(n.GetErrorString))dlsym(n.handle, "ncclGetErrorString");
  if (!n.GetUniqueId || !n.CommInitRank || !n.AllReduce) {
    n.handle = nullptr;
    return nullptr;
  }
  return &n;
}
void check_nccl(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) {
    Nccl* n = nccl();
    runtime_fail(std::string(what) + ": " +
                 (n && n->GetErrorString ? n->GetErrorString(r) : std::to_string(r)));
  }
}

}  // namespace

namespace tb {
void set_last_error(const char* message) { g_error = message; }
bool poisoned() {
  std::lock_guard<std::mutex> lock(g_mutex);
  return g_state == TB_POISONED;
}
void poison_library(const char* why) {
  g_error = why;
  poison(why);
}
}  // namespace tb

struct tb_instance;

struct tb_params {
  int device = 0;
  bool bf16 = false;  // the plan's network holds bf16 numbers: uploads round
  void* base = nullptr;
  std::vector<float*> slot;
  std::vector<int64_t> count;
  ~tb_params() {
    if (base) cudaFree(base);
  }
};

struct tb_comm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  // Abort rather than destroy: a communicator captured into a plan's graph may
  // still have work queued, and teardown must not wait on peers.
  ~tb_comm() {
    if (!comm || !nccl()) return;
    if (nccl()->CommAbort) nccl()->CommAbort(comm);
    else if (nccl()->CommDestroy) nccl()->CommDestroy(comm);
  }
};

struct tb_optimizer {
  tb_instance* plan = nullptr;  // the plan's main instance
  tb_params* params = nullptr;
  tb_optimizer_desc desc{};
  std::vector<int32_t> slots;
  std::vector<int> grad_buffers;       // plan buffer ids
  std::vector<tb::OptEntry> host_entries;
  tb::OptEntry* entries = nullptr;     // device table
  tb::OptEntry* custom = nullptr;      // device table for caller-given gradients
  float* state = nullptr;              // moments (Adam): first then second per slot
  float* scalars = nullptr;            // beta powers and corrections, learning rate
  bool bf16 = false;                   // the plan's parameters are bf16 numbers
  int64_t total = 0;
  std::vector<int64_t> state_offset;   // per entry
  ~tb_optimizer() {
    if (entries) cudaFree(entries);
    if (custom) cudaFree(custom);
    if (state) cudaFree(state);
    if (scalars) cudaFree(scalars);
  }
};

// 1 - beta (adam.rs:46-47) in the parameters' element type.
float optimizer_share(const tb_optimizer* o, float beta) {
  const float s = 1.0f - beta;
  return o->bf16 ? tb::round_bf16(s) : s;
}

// Per-run state of a plan: streams, arena, input buffers and the captured
// graph.  A plan owns a main instance (used by tb_plan_run, the optimizer and
// the communicator) and a pool that tb_run_begin draws from, so that runs of
// one compiled plan proceed concurrently from several threads, each on its own
// stream and arena.
struct tb_instance {
  tb_plan* owner = nullptr;
  tb::Program* prog = nullptr;         // the plan's (shared, immutable after compile)
  int device = 0;
  std::vector<CUfunction> fn;          // the plan's emitted kernels, per kernel
  cudaStream_t stream = nullptr, comm_stream = nullptr, side_stream = nullptr;
  char* arena = nullptr;
  std::vector<void*> own;              // input/leaf allocations
  std::vector<void*> buffer_ptr;       // resolved device pointer per buffer id
  std::vector<std::vector<void*>> kparams;
  tb_params* bound = nullptr;
  cudaGraphExec_t graph = nullptr;
  bool graph_dirty = true;
  tb::StreamK stream_k;                // the GEMMs' stream-K scratch (with any GEMM)
  tb_optimizer* optimizer = nullptr;
  tb_comm* comm = nullptr;
  int64_t bucket_bytes = 0;
  int reduction = TB_REDUCTION_NCCL;
  float* gather = nullptr;             // [world][bucket] shard gradients (tree reduction)
  int64_t gather_floats = 0;
  std::vector<cudaEvent_t> events;
  // Staged feeds: a host feed is copied on its own stream into one of two
  // staging buffers, overlapping the previous run's kernels; the run then
  // takes it with a device-to-device copy on its own stream.
  cudaStream_t copy_stream = nullptr;
  char* staging[2] = {nullptr, nullptr};
  int64_t staging_bytes = 0;
  cudaEvent_t staged[2] = {nullptr, nullptr}, consumed[2] = {nullptr, nullptr};
  uint64_t runs = 0;
  int64_t launches = 0;
  ~tb_instance() {
    if (stream) cudaStreamSynchronize(stream);
    if (gather) cudaFree(gather);
    if (graph) cudaGraphExecDestroy(graph);
    for (auto e : events) cudaEventDestroy(e);
    if (copy_stream) cudaStreamSynchronize(copy_stream);
    for (int k = 0; k < 2; ++k) {
      if (staging[k]) cudaFree(staging[k]);
      if (staged[k]) cudaEventDestroy(staged[k]);
      if (consumed[k]) cudaEventDestroy(consumed[k]);
    }
    if (copy_stream) cudaStreamDestroy(copy_stream);
    if (arena) cudaFree(arena);
    if (stream_k.workspace) cudaFree(stream_k.workspace);
    if (stream_k.flags) cudaFree(stream_k.flags);
    for (void* p : own) cudaFree(p);
    if (stream) cudaStreamDestroy(stream);
    if (comm_stream) cudaStreamDestroy(comm_stream);
    if (side_stream) cudaStreamDestroy(side_stream);
  }
};

struct tb_plan {
  std::unique_ptr<tb::Program> prog;
  int device = 0;
  CUmodule module = nullptr;
  std::vector<CUfunction> fn;
  std::unique_ptr<tb_instance> main;
  std::mutex pool_mutex;
  std::vector<std::unique_ptr<tb_instance>> pool;
  std::vector<tb_instance*> idle;
};

// A run drawn from the plan's pool (the reference's Run): its values stay
// readable until it is released.
struct tb_run {
  tb_plan* plan = nullptr;
  tb_instance* inst = nullptr;
};

namespace {

int resolve_node(const tb::Program& P, int64_t node) {
  if (node < 0 || node >= (int64_t)P.nodes.size()) throw Failure(TB_INVALID, "node out of range");
  int n = (int)node;
  while (P.info[n].alias >= 0) n = P.info[n].alias;
  return n;
}

int readable_buffer(const tb::Program& P, int64_t node) {
  int n = resolve_node(P, node);
  const tb::Info& f = P.info[n];
  if (!P.nodes[n].readable || !f.materialized || (f.owner != n && f.seed_of < 0))
    throw Failure(TB_INVALID, "node " + std::to_string(node) + " is not a readable value of the plan");
  return f.buf;
}

void bind_params(tb_instance* plan, tb_params* params) {
  tb::Program& P = *plan->prog;
  if (plan->bound == params) return;
  for (size_t b = 0; b < P.buffers.size(); ++b) {
    const tb::Buffer& buf = P.buffers[b];
    if (buf.storage != tb::Storage::Parameter) continue;
    if (!params || buf.slot >= (int)params->slot.size())
      throw Failure(TB_INVALID, "parameters do not cover the plan's parameter slots");
    if (params->count[buf.slot] * 4 != buf.bytes)
      throw Failure(TB_INVALID, "parameter slot size disagrees with the plan");
    plan->buffer_ptr[b] = params->slot[buf.slot];
  }
  plan->kparams.assign(P.kernels.size(), {});
  for (size_t k = 0; k < P.kernels.size(); ++k) {
    const tb::Kernel& K = P.kernels[k];
    for (int b : K.params) plan->kparams[k].push_back(plan->buffer_ptr[b]);
  }
  plan->bound = params;
  plan->graph_dirty = true;
}

float* fp(tb_instance* plan, int b) { return (float*)plan->buffer_ptr[b]; }
int* ip(tb_instance* plan, int b) { return (int*)plan->buffer_ptr[b]; }

// gradient ranges of the attached optimizer, issued after their last writer
struct Bucket {
  int after_kernel;
  char* begin;
  int64_t bytes;
};

std::vector<Bucket> gradient_buckets(tb_instance* plan) {
  std::vector<Bucket> out;
  if (!plan->optimizer || !plan->comm) return out;
  tb::Program& P = *plan->prog;
  struct Span {
    char* begin;
    int64_t bytes;
    int writer;
  };
  std::vector<Span> spans;
  for (int b : plan->optimizer->grad_buffers) {
    const tb::Buffer& buf = P.buffers[b];
    int writer = -1;
    for (size_t k = 0; k < P.kernels.size(); ++k)
      for (int w : P.kernels[k].writes)
        if (w == b) writer = std::max(writer, (int)k);
    spans.push_back({(char*)plan->buffer_ptr[b], buf.bytes, writer});
  }
  std::sort(spans.begin(), spans.end(), [](const Span& a, const Span& b) { return a.begin < b.begin; });
  // merge neighbours (the arena packs readable values contiguously in write order)
  std::vector<Span> merged;
  for (auto& s : spans) {
    if (!merged.empty()) {
      Span& m = merged.back();
      int64_t gap = s.begin - (m.begin + m.bytes);
      if (gap >= 0 && gap < 256 && m.bytes < plan->bucket_bytes) {
        m.bytes = s.begin + s.bytes - m.begin;
        m.writer = std::max(m.writer, s.writer);
        continue;
      }
    }
    merged.push_back(s);
  }
  for (auto& m : merged) out.push_back({m.writer, m.begin, m.bytes});
  return out;
}

int64_t launch_kernel(tb_instance* plan, size_t k, cudaStream_t stream) {
  tb::Program& P = *plan->prog;
  const tb::Kernel& K = P.kernels[k];
  int64_t launches = 0;
  switch (K.type) {
    case tb::KType::GEMM: {
      tb::Operand a, b;
      a.hi = fp(plan, K.a_hi);
      a.lo = K.a_lo >= 0 ? fp(plan, K.a_lo) : nullptr;  // none: raw f32 operand
      a.mn = K.a_mn;
      a.ld = K.a_ld;
      a.rows = K.a_rows;
      b.hi = fp(plan, K.b_hi);
      b.lo = K.b_lo >= 0 ? fp(plan, K.b_lo) : nullptr;
      b.mn = K.b_mn;
      b.ld = K.b_ld;
      b.rows = K.b_rows;
      tb::launch_gemm(a, b, fp(plan, K.out), K.partial >= 0 ? fp(plan, K.partial) : nullptr,
                      (int)K.passes, K.batch, K.m, K.n, K.kp, stream, &plan->stream_k);
      launches += 1;
      break;
    }
    case tb::KType::SORT:
      tb::launch_selection_sort(ip(plan, K.out), ip(plan, K.keys), ip(plan, K.vals),
                                ip(plan, K.tmp_keys), ip(plan, K.tmp_vals), ip(plan, K.counts),
                                ip(plan, K.rstart), ip(plan, K.rend), K.count, K.rows,
                                (int)K.passes, K.tiles, stream);
      launches += 2 + 3 * K.passes;
      break;
    case tb::KType::SEGSUM:
      tb::launch_segment_sum(fp(plan, K.partial), ip(plan, K.rstart), ip(plan, K.rend),
                             fp(plan, K.final_out), K.rows, K.final_width, K.count, stream);
      launches += 1;
      break;
    case tb::KType::FINAL:
      if (!K.final_parts.empty()) {
        tb::FinalSet set{};
        set.count = (int)K.final_parts.size();
        set.start[0] = 0;
        for (int e = 0; e < set.count; ++e) {
          set.part[e] = fp(plan, K.final_parts[e]);
          set.out[e] = fp(plan, K.final_outs[e]);
          set.width[e] = K.final_widths[e];
          set.start[e + 1] = set.start[e] + (int)((K.final_widths[e] + 7) / 8);
        }
        tb::launch_final_sum_multi(set, K.final_blocks, stream);
      } else {
        tb::launch_final_sum(fp(plan, K.partial), fp(plan, K.final_out), K.final_blocks,
                             K.final_width, stream);
      }
      launches += 1;
      break;
    default: {
      // programmatic stream serialization: the emitted kernels begin with
      // griddepcontrol.wait, so this launch may overlap the previous kernel's tail
      void* args[] = {plan->kparams[k].data()};
      CUlaunchAttribute attr;
      attr.id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
      attr.value.programmaticStreamSerializationAllowed = 1;
      CUlaunchConfig cfg = {};
      cfg.gridDimX = (unsigned)K.grid;
      cfg.gridDimY = cfg.gridDimZ = 1;
      cfg.blockDimX = (unsigned)K.block;
      cfg.blockDimY = cfg.blockDimZ = 1;
      cfg.sharedMemBytes = (unsigned)K.smem;
      cfg.hStream = stream;
      cfg.attrs = &attr;
      cfg.numAttrs = tb::pdl_enabled() ? 1 : 0;
      check(g_driver.LaunchKernelEx(&cfg, plan->fn[k], args, nullptr), "cuLaunchKernelEx");
      launches += 1;
    }
  }
  check(cudaGetLastError(), "kernel launch");
  return launches;
}

void enqueue_program(tb_instance* plan, cudaStream_t stream) {
  tb::Program& P = *plan->prog;
  std::vector<Bucket> buckets = gradient_buckets(plan);
  int64_t launches = 0;
  size_t next_event = 0;
  auto event = [&]() {
    if (next_event == plan->events.size()) {
      cudaEvent_t e;
      check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
      plan->events.push_back(e);
    }
    return plan->events[next_event++];
  };
  bool comm_used = false;
  // side kernels (selection sorts) fork off at the start; the main stream
  // joins them at P.side_join, the first kernel that uses what they wrote --
  // the arena keeps every side buffer allocated until that kernel
  bool forked = false, joined = true;
  for (size_t k = 0; k < P.kernels.size(); ++k) {
    const tb::Kernel& K = P.kernels[k];
    if (K.side) {
      if (!forked) {
        cudaEvent_t e = event();
        check(cudaEventRecord(e, stream), "cudaEventRecord");
        check(cudaStreamWaitEvent(plan->side_stream, e, 0), "cudaStreamWaitEvent");
        forked = true;
        joined = false;
      }
      launches += launch_kernel(plan, k, plan->side_stream);
      continue;
    }
    if (!joined && (int)k >= P.side_join) {
      cudaEvent_t e = event();
      check(cudaEventRecord(e, plan->side_stream), "cudaEventRecord");
      check(cudaStreamWaitEvent(stream, e, 0), "cudaStreamWaitEvent");
      joined = true;
    }
    launches += launch_kernel(plan, k, stream);
    for (const Bucket& b : buckets) {
      if (b.after_kernel != (int)k) continue;
      cudaEvent_t e = event();
      check(cudaEventRecord(e, stream), "cudaEventRecord");
      check(cudaStreamWaitEvent(plan->comm_stream, e, 0), "cudaStreamWaitEvent");
      if (plan->reduction == TB_REDUCTION_TREE) {
        // every rank gathers all shards' gradients and sums them in tree_sum's order
        check_nccl(nccl()->AllGather(b.begin, plan->gather, b.bytes / 4, ncclFloat32,
                                     plan->comm->comm, plan->comm_stream),
                   "ncclAllGather");
        tb::launch_tree_sum(plan->gather, plan->comm->world, b.bytes / 4, (float*)b.begin,
                            plan->comm_stream);
        launches += 1;
      } else {
        check_nccl(nccl()->AllReduce(b.begin, b.begin, b.bytes / 4, ncclFloat32, ncclSum,
                                     plan->comm->comm, plan->comm_stream),
                   "ncclAllReduce");
      }
      comm_used = true;
    }
  }
  if (comm_used) {
    cudaEvent_t e = event();
    check(cudaEventRecord(e, plan->comm_stream), "cudaEventRecord");
    check(cudaStreamWaitEvent(stream, e, 0), "cudaStreamWaitEvent");
  }
  if (plan->optimizer) {
    tb_optimizer* o = plan->optimizer;
    if (o->desc.kind != TB_OPTIMIZER_SGD) {
      tb::launch_adam_scalars(o->scalars, o->desc.beta1, o->desc.beta2, o->bf16, stream);
      launches += 1;
    }
    tb::launch_optimizer(o->entries, (int)o->host_entries.size(), o->total, o->scalars,
                         o->scalars + 4, o->desc.kind, o->desc.beta1, o->desc.beta2,
                         optimizer_share(o, o->desc.beta1), optimizer_share(o, o->desc.beta2),
                         o->desc.epsilon, o->desc.decay, o->desc.gradient_scale, o->bf16,
                         stream);
    launches += 1;
    check(cudaGetLastError(), "optimizer launch");
  }
  plan->launches = launches;
}

void run_plan(tb_instance* plan);

void setup_instance(tb_plan* owner, tb_instance* plan) {
  tb::Program& P = *owner->prog;
  plan->owner = owner;
  plan->prog = owner->prog.get();
  plan->device = owner->device;
  plan->fn = owner->fn;
  check(cudaStreamCreateWithFlags(&plan->stream, cudaStreamNonBlocking), "cudaStreamCreate");
  check(cudaStreamCreateWithFlags(&plan->comm_stream, cudaStreamNonBlocking), "cudaStreamCreate");
  check(cudaStreamCreateWithFlags(&plan->side_stream, cudaStreamNonBlocking), "cudaStreamCreate");
  plan->buffer_ptr.assign(P.buffers.size(), nullptr);
  int64_t input_bytes = 0;
  for (int b : P.input_buffer)
    if (b >= 0) input_bytes += (P.buffers[b].bytes + 255) / 256 * 256;
  if (input_bytes > 0) {
    check(cudaStreamCreateWithFlags(&plan->copy_stream, cudaStreamNonBlocking), "cudaStreamCreate");
    for (int k = 0; k < 2; ++k) {
      check(cudaMalloc((void**)&plan->staging[k], input_bytes), "cudaMalloc(staging)");
      check(cudaEventCreateWithFlags(&plan->staged[k], cudaEventDisableTiming), "cudaEventCreate");
      check(cudaEventCreateWithFlags(&plan->consumed[k], cudaEventDisableTiming), "cudaEventCreate");
    }
    plan->staging_bytes = input_bytes;
  }
  if (P.arena_bytes > 0) check(cudaMalloc((void**)&plan->arena, P.arena_bytes), "cudaMalloc(arena)");
  bool has_gemm = false;
  for (const tb::Kernel& K : P.kernels) has_gemm = has_gemm || K.type == tb::KType::GEMM;
  if (has_gemm) {
    // used only inside one GEMM launch at a time on this instance's stream;
    // every launch leaves the flags zero again
    check(cudaMalloc((void**)&plan->stream_k.workspace, tb::kStreamKWorkspaceBytes),
          "cudaMalloc(stream-K workspace)");
    check(cudaMalloc((void**)&plan->stream_k.flags, tb::kStreamKFlagBytes),
          "cudaMalloc(stream-K flags)");
    check(cudaMemsetAsync(plan->stream_k.flags, 0, tb::kStreamKFlagBytes, plan->stream),
          "cudaMemset(stream-K flags)");
  }
  for (size_t b = 0; b < P.buffers.size(); ++b) {
    tb::Buffer& buf = P.buffers[b];
    const tb::Node* node = buf.node >= 0 ? &P.nodes[buf.node] : nullptr;
    switch (buf.storage) {
      case tb::Storage::Arena:
        if (buf.first >= 0) plan->buffer_ptr[b] = plan->arena + buf.offset;
        break;
      case tb::Storage::Parameter:
        break;
      case tb::Storage::Input:
      case tb::Storage::InputIndices:
      case tb::Storage::Leaf:
      case tb::Storage::LeafIndices: {
        void* p = nullptr;
        check(cudaMalloc(&p, std::max<int64_t>(buf.bytes, 16)), "cudaMalloc(source)");
        plan->own.push_back(p);
        plan->buffer_ptr[b] = p;
        const void* init = nullptr;
        if (buf.storage == tb::Storage::Leaf || buf.storage == tb::Storage::Input)
          init = node->dense;
        else
          init = node->indices;
        if (init) {
          check(cudaMemcpy(p, init, buf.bytes, cudaMemcpyHostToDevice), "upload source");
        } else if (buf.storage == tb::Storage::Input && node->payload == TB_PAYLOAD_CONSTANT) {
          // an input whose initial payload is one value spread over its shape
          // (a dropout mask before its first feed) starts as that value
          std::vector<float> filled((size_t)(buf.bytes / 4), node->constant);
          check(cudaMemcpy(p, filled.data(), buf.bytes, cudaMemcpyHostToDevice), "upload source");
        } else {
          check(cudaMemset(p, 0, buf.bytes), "cudaMemset(source)");
        }
        if ((buf.storage == tb::Storage::Leaf || buf.storage == tb::Storage::LeafIndices) && !init)
          throw Failure(TB_INVALID, "leaf without payload");
        break;
      }
    }
  }
}

void instantiate(tb_plan* plan) {
  tb::Program& P = *plan->prog;
  check(cudaGetDevice(&plan->device), "cudaGetDevice");
  check(cudaFree(nullptr), "context init");
  plan->module = compile_module(P.source, plan->device);
  plan->fn.assign(P.kernels.size(), nullptr);
  for (size_t k = 0; k < P.kernels.size(); ++k) {
    const tb::Kernel& K = P.kernels[k];
    if (K.name.empty()) continue;
    check(g_driver.ModuleGetFunction(&plan->fn[k], plan->module, K.name.c_str()), "cuModuleGetFunction");
  }
  plan->main.reset(new tb_instance());
  setup_instance(plan, plan->main.get());
}

// Copies the feeds into the instance's input buffers and launches its graph.
void start_run(tb_instance* plan, tb_params* params, int32_t feed_count, const tb_feed* feeds) {
  tb::Program& P = *plan->prog;
  bind_params(plan, params);
  // host feeds go through staging slot `k`, free again once the run two
  // before this one has taken its copy (the `consumed` event)
  const int k = (int)(plan->runs & 1);
  bool any_staged = false;
  int64_t offset = 0;
  for (int32_t f = 0; f < feed_count; ++f) {
    const tb_feed& feed = feeds[f];
    if (feed.slot < 0 || feed.slot >= P.input_slots)
      throw Failure(TB_INVALID, "fed slot is not an input of the plan");
    int b = P.input_buffer[feed.slot];
    if (b < 0) continue;  // an input the plan does not read
    const tb::Buffer& buf = P.buffers[b];
    const void* src = buf.storage == tb::Storage::InputIndices ? (const void*)feed.indices
                                                               : (const void*)feed.dense;
    if (!src) throw Failure(TB_INVALID, "feed of the wrong payload kind");
    if (feed.on_device || !plan->copy_stream ||
        offset + buf.bytes > plan->staging_bytes) {
      check(cudaMemcpyAsync(plan->buffer_ptr[b], src, buf.bytes,
                            feed.on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                            plan->stream),
            "feed copy");
      continue;
    }
    if (!any_staged) {
      check(cudaStreamWaitEvent(plan->copy_stream, plan->consumed[k], 0), "wait staging");
      any_staged = true;
    }
    check(cudaMemcpyAsync(plan->staging[k] + offset, src, buf.bytes, cudaMemcpyHostToDevice,
                          plan->copy_stream),
          "feed copy");
    offset += (buf.bytes + 255) / 256 * 256;
  }
  if (any_staged) {
    check(cudaEventRecord(plan->staged[k], plan->copy_stream), "record staged");
    check(cudaStreamWaitEvent(plan->stream, plan->staged[k], 0), "wait staged");
    offset = 0;
    for (int32_t f = 0; f < feed_count; ++f) {
      const tb_feed& feed = feeds[f];
      int b = P.input_buffer[feed.slot];
      if (b < 0) continue;
      const tb::Buffer& buf = P.buffers[b];
      if (feed.on_device || offset + buf.bytes > plan->staging_bytes) continue;
      check(cudaMemcpyAsync(plan->buffer_ptr[b], plan->staging[k] + offset, buf.bytes,
                            cudaMemcpyDeviceToDevice, plan->stream),
            "feed copy");
      offset += (buf.bytes + 255) / 256 * 256;
    }
    check(cudaEventRecord(plan->consumed[k], plan->stream), "record consumed");
  }
  plan->runs++;
  run_plan(plan);
}

void read_value(tb_instance* plan, int64_t node, float* host, int64_t count) {
  int b = readable_buffer(*plan->prog, node);
  if (count * 4 != plan->prog->buffers[b].bytes) throw Failure(TB_INVALID, "read size mismatch");
  check(cudaMemcpyAsync(host, plan->buffer_ptr[b], count * 4, cudaMemcpyDeviceToHost,
                        plan->stream),
        "read");
  check(cudaStreamSynchronize(plan->stream), "cudaStreamSynchronize");
  // a bf16 network's values are bf16: a value a library kernel wrote (a GEMM,
  // a column final, a segment sum) holds its f32 accumulation, rounded here
  if (plan->prog->bf16)
    for (int64_t i = 0; i < count; ++i) host[i] = tb::round_bf16(host[i]);
}

void run_plan(tb_instance* plan) {
  if (plan->graph_dirty && plan->comm && plan->reduction == TB_REDUCTION_TREE) {
    // the gather buffer is allocated before capture (no allocation while capturing)
    if (plan->comm->world > 64) throw Failure(TB_INVALID, "tree reduction supports at most 64 ranks");
    int64_t most = 0;
    for (const Bucket& b : gradient_buckets(plan)) most = std::max<int64_t>(most, b.bytes / 4);
    const int64_t need = most * plan->comm->world;
    if (need > plan->gather_floats) {
      if (plan->gather) cudaFree(plan->gather);
      plan->gather = nullptr;
      plan->gather_floats = 0;
      check(cudaMalloc((void**)&plan->gather, need * 4), "cudaMalloc(gather)");
      plan->gather_floats = need;
    }
  }
  if (plan->graph_dirty) {
    if (plan->graph) {
      cudaGraphExecDestroy(plan->graph);
      plan->graph = nullptr;
    }
    cudaGraph_t g;
    check(cudaStreamBeginCapture(plan->stream, cudaStreamCaptureModeThreadLocal), "BeginCapture");
    try {
      enqueue_program(plan, plan->stream);
    } catch (...) {
      cudaStreamEndCapture(plan->stream, &g);
      throw;
    }
    check(cudaStreamEndCapture(plan->stream, &g), "EndCapture");
    check(cudaGraphInstantiate(&plan->graph, g, 0), "cudaGraphInstantiate");
    cudaGraphDestroy(g);
    plan->graph_dirty = false;
  }
  check(cudaGraphLaunch(plan->graph, plan->stream), "cudaGraphLaunch");
}

}  // namespace

namespace {
void json_str(std::ostringstream& o, const std::string& s) {
  o << '"';
  for (char c : s) {
    switch (c) {
      case '"': o << "\\\""; break;
      case '\\': o << "\\\\"; break;
      case '\n': o << "\\n"; break;
      case '\t': o << "\\t"; break;
      default:
        if ((unsigned char)c < 0x20) {
          char b[8];
          snprintf(b, sizeof b, "\\u%04x", c);
          o << b;
        } else {
          o << c;
        }
    }
  }
  o << '"';
}

template <class T>
void json_list(std::ostringstream& o, const std::vector<T>& v) {
  o << '[';
  for (size_t i = 0; i < v.size(); ++i) o << (i ? "," : "") << v[i];
  o << ']';
}

}  // namespace

extern "C" {

const char* tb_last_error(void) { return g_error.c_str(); }

int tb_status(char* message, size_t capacity) {
  int s = ensure_ready();
  std::string m;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    s = g_state;
    m = g_status_message;
  }
  if (message && capacity) {
    snprintf(message, capacity, "%s", m.c_str());
  }
  return s;
}

int tb_plan_compile(const tb_plan_desc* desc, tb_plan** out) {
  return guarded([&]() {
    auto prog = tb::lower(desc);
    if (desc->numerics == TB_NUMERICS_EXACT && !prog->exact) {
      g_error = "the plan holds kernels that are not bit-identical to the interpreter";
      return (int)TB_DECLINED;
    }
    std::unique_ptr<tb_plan> plan(new tb_plan());
    plan->prog = std::move(prog);
    instantiate(plan.get());
    *out = plan.release();
    return (int)TB_OK;
  });
}

void tb_plan_destroy(tb_plan* plan) {
  if (!plan) return;
  delete plan;  // each instance drains its stream before it frees its memory
}

int tb_plan_stats_get(const tb_plan* plan, tb_plan_stats* s) {
  return guarded([&]() {
    const tb::Program& P = *plan->prog;
    s->kernels = plan->main->launches ? plan->main->launches : (int64_t)P.kernels.size();
    s->arena_bytes = P.arena_bytes;
    s->unplanned_bytes = P.unplanned_bytes;
    s->fused_nodes = P.fused_nodes;
    s->bit_identical = P.exact ? 1 : 0;
    s->gemms = P.gemms;
    return (int)TB_OK;
  }, false);
}

int64_t tb_plan_describe(const tb_plan* plan, char* buffer, size_t capacity) {
  std::ostringstream o;
  const tb::Program& P = *plan->prog;
  for (size_t k = 0; k < P.kernels.size(); ++k) o << k << ": " << P.kernels[k].describe << "\n";
  o << "arena " << P.arena_bytes << " bytes (" << P.unplanned_bytes << " without reuse)\n";
  std::string s = o.str();
  if (buffer && capacity) snprintf(buffer, capacity, "%s", s.c_str());
  return (int64_t)s.size() + 1;
}

int tb_params_create(const tb_plan* plan, tb_params** out) {
  return guarded([&]() {
    const tb::Program& P = *plan->prog;
    std::unique_ptr<tb_params> p(new tb_params());
    check(cudaGetDevice(&p->device), "cudaGetDevice");
    p->bf16 = P.bf16;
    int slots = P.parameter_slots;
    std::vector<int64_t> offset(slots);
    int64_t total = 0;
    p->count.assign(slots, 0);
    for (int s = 0; s < slots; ++s) {
      int64_t c = 1;
      for (auto e : P.parameter_shapes[s]) c *= e;
      p->count[s] = c;
      offset[s] = total;
      total += (c + 63) / 64 * 64;
    }
    check(cudaMalloc(&p->base, std::max<int64_t>(total * 4, 256)), "cudaMalloc(parameters)");
    check(cudaMemset(p->base, 0, std::max<int64_t>(total * 4, 256)), "cudaMemset(parameters)");
    for (int s = 0; s < slots; ++s) p->slot.push_back((float*)p->base + offset[s]);
    *out = p.release();
    return (int)TB_OK;
  });
}

void tb_params_destroy(tb_params* params) { delete params; }

int tb_params_upload(tb_params* params, int32_t slot, const float* host, int64_t count) {
  return guarded([&]() {
    if (slot < 0 || slot >= (int)params->slot.size() || count != params->count[slot])
      throw Failure(TB_INVALID, "parameter slot or size mismatch");
    if (params->bf16) {
      // a bf16 network's parameters are bf16 numbers (payload/bf16.rs:39-55)
      std::vector<float> rounded(host, host + count);
      for (float& v : rounded) v = tb::round_bf16(v);
      check(cudaMemcpy(params->slot[slot], rounded.data(), count * 4, cudaMemcpyHostToDevice),
            "upload");
      return (int)TB_OK;
    }
    check(cudaMemcpy(params->slot[slot], host, count * 4, cudaMemcpyHostToDevice), "upload");
    return (int)TB_OK;
  });
}

int tb_params_download(const tb_params* params, int32_t slot, float* host, int64_t count) {
  return guarded([&]() {
    if (slot < 0 || slot >= (int)params->slot.size() || count != params->count[slot])
      throw Failure(TB_INVALID, "parameter slot or size mismatch");
    check(cudaDeviceSynchronize(), "sync");
    check(cudaMemcpy(host, params->slot[slot], count * 4, cudaMemcpyDeviceToHost), "download");
    return (int)TB_OK;
  });
}

int tb_plan_run(tb_plan* plan, tb_params* params, int32_t feed_count, const tb_feed* feeds) {
  return guarded([&]() {
    start_run(plan->main.get(), params, feed_count, feeds);
    return (int)TB_OK;
  });
}

int tb_plan_gradient_node(const tb_plan* plan, int64_t root, int64_t parameter, int64_t* node) {
  return guarded([&]() {
    auto it = plan->prog->gradient_of.find({(int)root, (int)parameter});
    if (it == plan->prog->gradient_of.end())
      throw Failure(TB_INVALID, "no gradient of that root with respect to that parameter: "
                                "compile with backward set, a scalar readable root and a "
                                "parameter node");
    *node = it->second;
    return (int)TB_OK;
  }, false);
}

// A kernel whose bounded wait expired recorded a code instead of hanging: the
// run's values are not to be trusted, which is a runtime failure (poisons).
static void check_device_flags() {
  const int g = tb::gemm_error(), s = tb::segment_error();
  if (g || s)
    runtime_fail("a device wait expired (gemm code " + std::to_string(g) + ", segment code " +
                 std::to_string(s) + ")");
}

int tb_plan_synchronize(tb_plan* plan) {
  return guarded([&]() {
    check(cudaStreamSynchronize(plan->main->stream), "cudaStreamSynchronize");
    check_device_flags();
    return (int)TB_OK;
  });
}

int tb_plan_read(tb_plan* plan, int64_t node, float* host, int64_t count) {
  return guarded([&]() {
    read_value(plan->main.get(), node, host, count);
    return (int)TB_OK;
  });
}

int tb_plan_read_async(tb_plan* plan, int64_t node, float* host, int64_t count) {
  return guarded([&]() {
    tb_instance* inst = plan->main.get();
    if (inst->prog->bf16)
      throw Failure(TB_INVALID, "tb_plan_read_async: a bf16 plan's reads round on the host");
    int b = readable_buffer(*inst->prog, node);
    if (count * 4 != inst->prog->buffers[b].bytes) throw Failure(TB_INVALID, "read size mismatch");
    check(cudaMemcpyAsync(host, inst->buffer_ptr[b], count * 4, cudaMemcpyDeviceToHost,
                          inst->stream),
          "read");
    return (int)TB_OK;
  });
}

int tb_plan_device_pointer(tb_plan* plan, int64_t node, const float** device) {
  return guarded([&]() {
    int b = readable_buffer(*plan->prog, node);
    *device = (const float*)plan->main->buffer_ptr[b];
    return (int)TB_OK;
  });
}

void* tb_plan_stream(tb_plan* plan) { return plan ? (void*)plan->main->stream : nullptr; }

int tb_run_begin(tb_plan* plan, tb_params* params, int32_t feed_count, const tb_feed* feeds,
                 tb_run** out) {
  return guarded([&]() {
    tb_instance* inst = nullptr;
    {
      std::lock_guard<std::mutex> lock(plan->pool_mutex);
      if (!plan->idle.empty()) {
        inst = plan->idle.back();
        plan->idle.pop_back();
      } else {
        std::unique_ptr<tb_instance> fresh(new tb_instance());
        setup_instance(plan, fresh.get());
        inst = fresh.get();
        plan->pool.push_back(std::move(fresh));
      }
    }
    std::unique_ptr<tb_run> run(new tb_run());
    run->plan = plan;
    run->inst = inst;
    try {
      start_run(inst, params, feed_count, feeds);
    } catch (...) {
      std::lock_guard<std::mutex> lock(plan->pool_mutex);
      plan->idle.push_back(inst);
      throw;
    }
    *out = run.release();
    return (int)TB_OK;
  });
}

int tb_run_synchronize(tb_run* run) {
  return guarded([&]() {
    check(cudaStreamSynchronize(run->inst->stream), "cudaStreamSynchronize");
    check_device_flags();
    return (int)TB_OK;
  });
}

int tb_run_read(tb_run* run, int64_t node, float* host, int64_t count) {
  return guarded([&]() {
    read_value(run->inst, node, host, count);
    return (int)TB_OK;
  });
}

int tb_run_device_pointer(tb_run* run, int64_t node, const float** device) {
  return guarded([&]() {
    int b = readable_buffer(*run->plan->prog, node);
    *device = (const float*)run->inst->buffer_ptr[b];
    return (int)TB_OK;
  });
}

void* tb_run_stream(tb_run* run) { return run ? (void*)run->inst->stream : nullptr; }

void tb_run_release(tb_run* run) {
  if (!run) return;
  {
    // the next run on this instance is ordered after this one by its stream
    std::lock_guard<std::mutex> lock(run->plan->pool_mutex);
    run->plan->idle.push_back(run->inst);
  }
  delete run;
}

int tb_optimizer_create(tb_plan* owner, tb_params* params, const tb_optimizer_desc* desc,
                        int32_t count, const int32_t* slots, const int64_t* gradient_nodes,
                        tb_optimizer** out) {
  return guarded([&]() {
    tb_instance* plan = owner->main.get();
    if (desc->kind < 0 || desc->kind > 2) throw Failure(TB_INVALID, "unknown optimizer kind");
    bind_params(plan, params);
    std::unique_ptr<tb_optimizer> o(new tb_optimizer());
    o->plan = plan;
    o->params = params;
    o->desc = *desc;
    o->bf16 = plan->prog->bf16;
    if (o->bf16) {
      // Adam<Bf16> and the rate hold bf16 scalars (neural/adam.rs:40-56)
      if (desc->gradient_scale != 1.0f)
        throw Failure(TB_DECLINED, "a bf16 step takes no gradient scale");
      for (float* h : {&o->desc.learning_rate, &o->desc.beta1, &o->desc.beta2,
                       &o->desc.epsilon, &o->desc.decay})
        *h = tb::round_bf16(*h);
    }
    int64_t total = 0;
    for (int32_t i = 0; i < count; ++i) {
      int slot = slots[i];
      if (slot < 0 || slot >= (int)params->slot.size()) throw Failure(TB_INVALID, "bad slot");
      int b = readable_buffer(*plan->prog, gradient_nodes[i]);
      if (plan->prog->buffers[b].bytes != params->count[slot] * 4)
        throw Failure(TB_INVALID, "gradient and parameter sizes differ");
      tb::OptEntry e{};
      e.p = params->slot[slot];
      e.g = (const float*)plan->buffer_ptr[b];
      e.count = params->count[slot];
      e.start = total;
      e.decay = plan->prog->parameter_shapes[slot].size() >= 2 ? 1 : 0;
      o->slots.push_back(slot);
      o->grad_buffers.push_back(b);
      o->host_entries.push_back(e);
      total += e.count;
    }
    o->total = total;
    check(cudaMalloc((void**)&o->scalars, 8 * 4), "cudaMalloc(scalars)");
    float init[8] = {1.0f, 1.0f, 0.0f, 0.0f, desc->learning_rate, 0, 0, 0};
    check(cudaMemcpy(o->scalars, init, sizeof init, cudaMemcpyHostToDevice), "upload scalars");
    if (desc->kind != TB_OPTIMIZER_SGD && total > 0) {
      check(cudaMalloc((void**)&o->state, total * 2 * 4), "cudaMalloc(moments)");
      check(cudaMemset(o->state, 0, total * 2 * 4), "cudaMemset(moments)");
      for (auto& e : o->host_entries) {
        e.m = o->state + e.start;
        e.v = o->state + total + e.start;
      }
    }
    if (!o->host_entries.empty()) {
      check(cudaMalloc((void**)&o->entries, o->host_entries.size() * sizeof(tb::OptEntry)),
            "cudaMalloc(entries)");
      check(cudaMemcpy(o->entries, o->host_entries.data(),
                       o->host_entries.size() * sizeof(tb::OptEntry), cudaMemcpyHostToDevice),
            "upload entries");
    }
    *out = o.release();
    return (int)TB_OK;
  });
}

void tb_optimizer_destroy(tb_optimizer* o) {
  if (!o) return;
  if (o->plan && o->plan->optimizer == o) {
    o->plan->optimizer = nullptr;
    o->plan->graph_dirty = true;
  }
  cudaDeviceSynchronize();
  delete o;
}

int tb_optimizer_set_learning_rate(tb_optimizer* o, float lr) {
  return guarded([&]() {
    o->desc.learning_rate = o->bf16 ? tb::round_bf16(lr) : lr;
    check(cudaMemcpyAsync(o->scalars + 4, &o->desc.learning_rate, 4, cudaMemcpyHostToDevice,
                          o->plan->stream),
          "upload learning rate");
    check(cudaStreamSynchronize(o->plan->stream), "sync");
    return (int)TB_OK;
  });
}

int tb_optimizer_step(tb_optimizer* o, const float* const* gradients, void* stream) {
  return guarded([&]() {
    cudaStream_t st = stream ? (cudaStream_t)stream : o->plan->stream;
    const tb::OptEntry* table = o->entries;
    if (gradients && !o->host_entries.empty()) {
      if (!o->custom)
        check(cudaMalloc((void**)&o->custom, o->host_entries.size() * sizeof(tb::OptEntry)),
              "cudaMalloc(entries)");
      std::vector<tb::OptEntry> e = o->host_entries;
      for (size_t i = 0; i < e.size(); ++i) {
        if (!gradients[i]) throw Failure(TB_INVALID, "missing gradient pointer");
        e[i].g = gradients[i];
      }
      // synchronous: the table is tiny and must not outlive this call's host copy
      check(cudaStreamSynchronize(st), "sync");
      check(cudaMemcpy(o->custom, e.data(), e.size() * sizeof(tb::OptEntry),
                       cudaMemcpyHostToDevice),
            "upload entries");
      table = o->custom;
    }
    if (o->desc.kind != TB_OPTIMIZER_SGD)
      tb::launch_adam_scalars(o->scalars, o->desc.beta1, o->desc.beta2, o->bf16, st);
    tb::launch_optimizer(table, (int)o->host_entries.size(), o->total, o->scalars, o->scalars + 4,
                         o->desc.kind, o->desc.beta1, o->desc.beta2,
                         optimizer_share(o, o->desc.beta1), optimizer_share(o, o->desc.beta2),
                         o->desc.epsilon, o->desc.decay, o->desc.gradient_scale, o->bf16, st);
    check(cudaGetLastError(), "optimizer launch");
    return (int)TB_OK;
  });
}

int tb_plan_attach_optimizer(tb_plan* owner, tb_optimizer* o) {
  return guarded([&]() {
    tb_instance* plan = owner->main.get();
    if (o && o->plan != plan) throw Failure(TB_INVALID, "optimizer belongs to another plan");
    plan->optimizer = o;
    plan->graph_dirty = true;
    return (int)TB_OK;
  });
}

int tb_optimizer_state(const tb_optimizer* o, int32_t slot, float* first, float* second,
                       int64_t count) {
  return guarded([&]() {
    if (!o->state) throw Failure(TB_INVALID, "optimizer has no moments");
    for (size_t i = 0; i < o->slots.size(); ++i) {
      if (o->slots[i] != slot) continue;
      const tb::OptEntry& e = o->host_entries[i];
      if (e.count != count) throw Failure(TB_INVALID, "size mismatch");
      check(cudaDeviceSynchronize(), "sync");
      check(cudaMemcpy(first, e.m, count * 4, cudaMemcpyDeviceToHost), "download");
      check(cudaMemcpy(second, e.v, count * 4, cudaMemcpyDeviceToHost), "download");
      return (int)TB_OK;
    }
    throw Failure(TB_INVALID, "slot not bound to the optimizer");
  });
}

int tb_optimizer_powers(const tb_optimizer* o, float powers[2]) {
  return guarded([&]() {
    if (!o->state) throw Failure(TB_INVALID, "optimizer has no moments");
    check(cudaDeviceSynchronize(), "sync");
    check(cudaMemcpy(powers, o->scalars, 2 * 4, cudaMemcpyDeviceToHost), "download");
    return (int)TB_OK;
  });
}

int tb_optimizer_restore(tb_optimizer* o, int32_t slot, const float* first, const float* second,
                         int64_t count) {
  return guarded([&]() {
    if (!o->state) throw Failure(TB_INVALID, "optimizer has no moments");
    for (size_t i = 0; i < o->slots.size(); ++i) {
      if (o->slots[i] != slot) continue;
      const tb::OptEntry& e = o->host_entries[i];
      if (e.count != count) throw Failure(TB_INVALID, "size mismatch");
      check(cudaDeviceSynchronize(), "sync");
      check(cudaMemcpy(e.m, first, count * 4, cudaMemcpyHostToDevice), "upload");
      check(cudaMemcpy(e.v, second, count * 4, cudaMemcpyHostToDevice), "upload");
      return (int)TB_OK;
    }
    throw Failure(TB_INVALID, "slot not bound to the optimizer");
  });
}

int tb_optimizer_restore_powers(tb_optimizer* o, const float powers[2]) {
  return guarded([&]() {
    if (!o->state) throw Failure(TB_INVALID, "optimizer has no moments");
    // s[0..1] are the powers the next step multiplies; s[2..3] their
    // corrections, recomputed by that step before use
    const float s[4] = {powers[0], powers[1], 1.0f - powers[0], 1.0f - powers[1]};
    check(cudaDeviceSynchronize(), "sync");
    check(cudaMemcpy(o->scalars, s, sizeof s, cudaMemcpyHostToDevice), "upload");
    return (int)TB_OK;
  });
}

int tb_comm_unique_id(uint8_t id[128]) {
  return guarded([&]() {
    Nccl* n = nccl();
    if (!n) throw Failure(TB_INITIALIZATION, "NCCL is not loadable");
    ncclUniqueId u;
    check_nccl(n->GetUniqueId(&u), "ncclGetUniqueId");
    memcpy(id, u.internal, 128);
    return (int)TB_OK;
  });
}

int tb_comm_init(int32_t rank, int32_t world, const uint8_t id[128], tb_comm** out) {
  return guarded([&]() {
    Nccl* n = nccl();
    if (!n) throw Failure(TB_INITIALIZATION, "NCCL is not loadable");
    std::unique_ptr<tb_comm> c(new tb_comm());
    ncclUniqueId u;
    memcpy(u.internal, id, 128);
    check_nccl(n->CommInitRank(&c->comm, world, u, rank), "ncclCommInitRank");
    c->rank = rank;
    c->world = world;
    *out = c.release();
    return (int)TB_OK;
  });
}

void tb_comm_destroy(tb_comm* comm) { delete comm; }

int tb_plan_attach_comm(tb_plan* owner, tb_comm* comm, int64_t bucket_bytes) {
  return guarded([&]() {
    tb_instance* plan = owner->main.get();
    if (plan->prog->bf16) throw Failure(TB_DECLINED, "the gradient exchange sums f32 gradients");
    plan->comm = comm;
    plan->bucket_bytes = bucket_bytes > 0 ? bucket_bytes : (int64_t)32 << 20;
    plan->graph_dirty = true;
    return (int)TB_OK;
  });
}

int tb_plan_set_reduction(tb_plan* owner, int32_t reduction) {
  return guarded([&]() {
    if (reduction != TB_REDUCTION_NCCL && reduction != TB_REDUCTION_TREE)
      throw Failure(TB_INVALID, "unknown reduction");
    if (reduction == TB_REDUCTION_TREE && (!nccl() || !nccl()->AllGather))
      throw Failure(TB_INITIALIZATION, "ncclAllGather is not loadable");
    if (owner->main->comm && owner->main->comm->world > 64)
      throw Failure(TB_INVALID, "tree reduction supports at most 64 ranks");
    owner->main->reduction = reduction;
    owner->main->graph_dirty = true;
    return (int)TB_OK;
  });
}

int tb_comm_allreduce(tb_comm* comm, float* device, int64_t count, void* stream) {
  return guarded([&]() {
    check_nccl(nccl()->AllReduce(device, device, count, ncclFloat32, ncclSum, comm->comm,
                                 (cudaStream_t)stream),
               "ncclAllReduce");
    return (int)TB_OK;
  });
}

// ---- internal hooks for CPU-side tests (not part of the public ABI): lowering
// and NVRTC compilation need no device.
int64_t tbx_lower_describe(const tb_plan_desc* desc, char* buffer, size_t capacity, int with_source) {
  try {
    auto prog = tb::lower(desc);
    std::ostringstream o;
    for (size_t k = 0; k < prog->kernels.size(); ++k) o << k << ": " << prog->kernels[k].describe << "\n";
    o << "arena " << prog->arena_bytes << " bytes (" << prog->unplanned_bytes << " without reuse)\n";
    o << "exact " << (prog->exact ? 1 : 0) << " fused " << prog->fused_nodes << "\n";
    if (prog->side_join >= 0) o << "side join " << prog->side_join << "\n";
    for (size_t b = 0; b < prog->buffers.size(); ++b) {
      const tb::Buffer& buf = prog->buffers[b];
      if (!buf.keep) continue;
      int writer = -1;
      for (size_t k = 0; k < prog->kernels.size(); ++k)
        for (int w : prog->kernels[k].writes)
          if (w == (int)b) writer = (int)k;
      o << "keep buffer " << b << " node " << buf.node << " offset " << buf.offset << " bytes "
        << buf.bytes << " writer " << writer << "\n";
    }
    // a value's buffer written by a kernel and read by no other kernel, and not
    // a result: a store nobody needs, or a round trip through memory inside its
    // own kernel (a kernel's parameter is listed as written when it writes it).
    // Scratch such as split-K partials is used inside its own launch and is not
    // listed.
    for (size_t b = 0; b < prog->buffers.size(); ++b) {
      const tb::Buffer& buf = prog->buffers[b];
      if (buf.keep || buf.node < 0) continue;
      std::set<int> writers, readers;
      for (size_t k = 0; k < prog->kernels.size(); ++k) {
        for (int w : prog->kernels[k].writes)
          if (w == (int)b) writers.insert((int)k);
        for (int r : prog->kernels[k].reads)
          if (r == (int)b) readers.insert((int)k);
      }
      if (!writers.empty() && readers.empty())
        o << "dead buffer " << b << " node " << buf.node << " bytes " << buf.bytes << "\n";
    }
    if (with_source) o << prog->source;
    std::string s = o.str();
    if (buffer && capacity) snprintf(buffer, capacity, "%s", s.c_str());
    return (int64_t)s.size() + 1;
  } catch (const std::exception& e) {
    g_error = e.what();
    return -1;
  }
}

// The lowered program as JSON, for the host-side kernel emulator of the
// tests: kernels in order with their buffers and launch shapes, the buffer
// table, the buffers of readable values, and the emitted source.
int64_t tbx_lower_json(const tb_plan_desc* desc, char* buffer, size_t capacity) {
  try {
    auto prog = tb::lower(desc);
    static const char* types[] = {"ew", "row", "reduce", "prep", "gemm", "sort", "scatter",
                                  "fold", "final", "segsum"};
    std::ostringstream o;
    o << "{\"bf16\":" << (prog->bf16 ? 1 : 0) << ",\"arena_bytes\":" << prog->arena_bytes
      << ",\"kernels\":[";
    for (size_t k = 0; k < prog->kernels.size(); ++k) {
      const tb::Kernel& K = prog->kernels[k];
      o << (k ? "," : "") << "{\"type\":\"" << types[(int)K.type] << "\",\"name\":";
      json_str(o, K.name);
      o << ",\"grid\":" << K.grid << ",\"block\":" << K.block << ",\"params\":";
      json_list(o, K.params);
      o << ",\"a_hi\":" << K.a_hi << ",\"a_lo\":" << K.a_lo << ",\"b_hi\":" << K.b_hi
        << ",\"b_lo\":" << K.b_lo << ",\"out\":" << K.out << ",\"batch\":" << K.batch
        << ",\"m\":" << K.m << ",\"n\":" << K.n << ",\"k\":" << K.k << ",\"kp\":" << K.kp
        << ",\"a_mn\":" << K.a_mn << ",\"b_mn\":" << K.b_mn << ",\"a_ld\":" << K.a_ld
        << ",\"b_ld\":" << K.b_ld << ",\"a_rows\":" << K.a_rows << ",\"b_rows\":" << K.b_rows
        << ",\"keys\":" << K.keys << ",\"vals\":" << K.vals << ",\"rstart\":" << K.rstart
        << ",\"rend\":" << K.rend << ",\"count\":" << K.count << ",\"rows\":" << K.rows
        << ",\"partial\":" << K.partial << ",\"final_out\":" << K.final_out
        << ",\"final_blocks\":" << K.final_blocks << ",\"final_width\":" << K.final_width
        << ",\"final_parts\":";
      json_list(o, K.final_parts);
      o << ",\"final_outs\":";
      json_list(o, K.final_outs);
      o << ",\"final_widths\":";
      json_list(o, K.final_widths);
      o << "}";
    }
    o << "],\"buffers\":[";
    for (size_t b = 0; b < prog->buffers.size(); ++b) {
      const tb::Buffer& B = prog->buffers[b];
      o << (b ? "," : "") << "{\"storage\":" << (int)B.storage << ",\"bytes\":" << B.bytes
        << ",\"slot\":" << B.slot << ",\"node\":" << B.node << ",\"offset\":" << B.offset
        << ",\"placed\":" << (B.first >= 0 ? 1 : 0) << "}";
    }
    o << "],\"readable\":{";
    bool first = true;
    for (size_t n = 0; n < prog->nodes.size(); ++n) {
      // as readable_buffer answers: through the alias of an expanded node
      const int r = resolve_node(*prog, (int64_t)n);
      const tb::Info& f = prog->info[r];
      if (!prog->nodes[r].readable || !f.materialized || (f.owner != r && f.seed_of < 0)) continue;
      o << (first ? "" : ",") << "\"" << n << "\":[" << f.buf << ",";
      json_list(o, prog->nodes[n].dims());
      o << "]";
      first = false;
    }
    o << "},\"gradients\":[";
    bool any = false;
    for (const auto& g : prog->gradient_of) {
      o << (any ? "," : "") << "[" << g.first.first << "," << g.first.second << "," << g.second
        << "]";
      any = true;
    }
    o << "],\"source\":";
    json_str(o, prog->source);
    o << "}";
    std::string s = o.str();
    if (buffer && capacity) snprintf(buffer, capacity, "%s", s.c_str());
    return (int64_t)s.size() + 1;
  } catch (const std::exception& e) {
    g_error = e.what();
    return -1;
  }
}

int tbx_nvrtc_check(const tb_plan_desc* desc) {
  try {
    auto prog = tb::lower(desc);
    nvrtcProgram p;
    if (nvrtcCreateProgram(&p, prog->source.c_str(), "check.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS)
      return TB_RUNTIME;
    const char* opts[] = {"-arch=sm_100a", "--fmad=false", "-prec-div=true", "-prec-sqrt=true",
                          "-ftz=false", "-std=c++17", "-default-device"};
    nvrtcResult r = nvrtcCompileProgram(p, 7, opts);
    if (r != NVRTC_SUCCESS) {
      size_t n = 0;
      nvrtcGetProgramLogSize(p, &n);
      std::string log(n, '\0');
      nvrtcGetProgramLog(p, &log[0]);
      g_error = log.substr(0, 4000);
    }
    nvrtcDestroyProgram(&p);
    return r == NVRTC_SUCCESS ? TB_OK : TB_INVALID;
  } catch (const std::exception& e) {
    g_error = e.what();
    return TB_INVALID;
  }
}

// Times each kernel of a bound plan on its own (after one warm launch):
// ms[k] = average of `reps` launches.  Returns the kernel count.
int64_t tbx_profile_kernels(tb_plan* owner, int reps, float* ms, int64_t capacity) {
  tb_instance* plan = owner->main.get();
  int rc = guarded([&]() {
    if (!plan->bound) throw Failure(TB_INVALID, "run the plan once before profiling");
    tb::Program& P = *plan->prog;
    cudaEvent_t a, b;
    check(cudaEventCreate(&a), "cudaEventCreate");
    check(cudaEventCreate(&b), "cudaEventCreate");
    for (size_t k = 0; k < P.kernels.size() && (int64_t)k < capacity; ++k) {
      launch_kernel(plan, k, plan->stream);
      check(cudaEventRecord(a, plan->stream), "record");
      for (int r = 0; r < reps; ++r) launch_kernel(plan, k, plan->stream);
      check(cudaEventRecord(b, plan->stream), "record");
      check(cudaEventSynchronize(b), "sync");
      float t = 0;
      cudaEventElapsedTime(&t, a, b);
      ms[k] = t / reps;
    }
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    return (int)TB_OK;
  });
  return rc == TB_OK ? (int64_t)plan->prog->kernels.size() : -1;
}

// Per-kernel facts for roofline accounting: type, gemm dims, bytes of the
// buffers it reads and writes.
int tbx_kernel_facts(tb_plan* plan, int64_t k, int64_t* facts) {
  return guarded([&]() {
    tb::Program& P = *plan->prog;
    const tb::Kernel& K = P.kernels.at(k);
    int64_t rd = 0, wr = 0;
    for (int b : K.reads) rd += P.buffers[b].bytes;
    for (int b : K.writes) wr += P.buffers[b].bytes;
    facts[0] = (int64_t)K.type;
    facts[1] = K.batch;
    facts[2] = K.m;
    facts[3] = K.n;
    facts[4] = K.k;
    facts[5] = rd;
    facts[6] = wr;
    facts[7] = K.grid;
    return (int)TB_OK;
  }, false);
}

// ---- per-task faces
int tb_gemm_f32(const float* a, int64_t a_len, const int64_t a_strides[2], const float* b,
                int64_t b_len, const int64_t b_strides[2], int64_t m, int64_t k, int64_t n,
                float* out);
int tb_map_f32(int32_t op, const float* in, int64_t count, float* out);

}  // extern "C"
