// B200 execution runtime for tensorjit kernel plans (C ABI declared in include/tj_b200.h).
//
// One Program owns: the loaded sm_100a modules, a device arena for the planned
// intermediates, a status word that kernels write when a bounded wait runs out,
// and (in graph mode) one instantiated CUDA graph of the whole kernel list.
//
// Per call the runtime resolves every kernel argument from its tj_argref
// (caller input, caller output, arena + offset, status word) into the kernel's
// single by-value parameter block, encodes any TMA descriptors against the
// resolved addresses, and launches with cuLaunchKernelEx on the caller's
// stream.  In graph mode a call only re-points the kernel nodes whose
// parameter block changed (cuGraphExecKernelNodeSetParams) and replays the
// graph: caller buffers are bound directly, never copied into static buffers.
//
// libcuda is opened with dlopen on first use, so the library loads (and its
// symbols can be listed) on a machine without a driver.
#include "../../include/tj_b200.h"

#include <cuda.h>
#include <dlfcn.h>
// NVTX ranges name every plan kernel on a profiler timeline (nsys / ncu --nvtx).  NVTX v3 is
// header-only: without a tool attached the calls return at once.
#include <nvtx3/nvToolsExt.h>

#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

// ---------------------------------------------------------------------------
// libcuda, loaded lazily
// ---------------------------------------------------------------------------
struct Driver {
  bool ok = false;
  std::string why;
#define TJ_FN(name) decltype(&::name) name = nullptr
  TJ_FN(cuInit);
  TJ_FN(cuDeviceGet);
  TJ_FN(cuDeviceGetCount);
  TJ_FN(cuDevicePrimaryCtxRetain);
  TJ_FN(cuDevicePrimaryCtxRelease_v2);
  TJ_FN(cuCtxPushCurrent_v2);
  TJ_FN(cuCtxPopCurrent_v2);
  TJ_FN(cuCtxSynchronize);
  TJ_FN(cuModuleLoadData);
  TJ_FN(cuModuleUnload);
  TJ_FN(cuModuleGetFunction);
  TJ_FN(cuFuncSetAttribute);
  TJ_FN(cuFuncGetParamInfo);
  TJ_FN(cuMemAlloc_v2);
  TJ_FN(cuMemFree_v2);
  TJ_FN(cuMemsetD32_v2);
  TJ_FN(cuMemcpyDtoH_v2);
  TJ_FN(cuLaunchKernelEx);
  TJ_FN(cuTensorMapEncodeTiled);
  TJ_FN(cuGraphCreate);
  TJ_FN(cuGraphAddKernelNode_v2);
  TJ_FN(cuGraphAddDependencies_v2);
  TJ_FN(cuGraphKernelNodeSetAttribute);
  TJ_FN(cuGraphInstantiateWithFlags);
  TJ_FN(cuGraphLaunch);
  TJ_FN(cuGraphExecKernelNodeSetParams_v2);
  TJ_FN(cuGraphExecDestroy);
  TJ_FN(cuGraphDestroy);
  TJ_FN(cuGetErrorString);
  TJ_FN(cuEventCreate);
  TJ_FN(cuEventDestroy_v2);
  TJ_FN(cuEventRecord);
  TJ_FN(cuEventSynchronize);
  TJ_FN(cuEventElapsedTime);
  TJ_FN(cuOccupancyMaxActiveClusters);
  TJ_FN(cuMemGetAddressRange_v2);
  TJ_FN(cuIpcGetMemHandle);
  TJ_FN(cuIpcOpenMemHandle_v2);
  TJ_FN(cuIpcCloseMemHandle);
#undef TJ_FN

  void load() {
    void* h = dlopen("libcuda.so.1", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libcuda.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      why = std::string("cannot load libcuda: ") + dlerror();
      return;
    }
    bool all = true;
#define TJ_SYM(name)                                                      \
  name = reinterpret_cast<decltype(name)>(dlsym(h, #name));               \
  if (!name) { all = false; why += std::string(" missing ") + #name; }
#define TJ_SYM_OPT(name) name = reinterpret_cast<decltype(name)>(dlsym(h, #name));
    TJ_SYM(cuInit) TJ_SYM(cuDeviceGet) TJ_SYM(cuDeviceGetCount) TJ_SYM(cuDevicePrimaryCtxRetain)
    TJ_SYM(cuDevicePrimaryCtxRelease_v2) TJ_SYM(cuCtxPushCurrent_v2) TJ_SYM(cuCtxPopCurrent_v2)
    TJ_SYM(cuCtxSynchronize) TJ_SYM(cuModuleLoadData) TJ_SYM(cuModuleUnload) TJ_SYM(cuModuleGetFunction)
    TJ_SYM(cuFuncSetAttribute) TJ_SYM_OPT(cuFuncGetParamInfo) TJ_SYM(cuMemAlloc_v2) TJ_SYM(cuMemFree_v2)
    TJ_SYM(cuMemsetD32_v2) TJ_SYM(cuMemcpyDtoH_v2) TJ_SYM(cuLaunchKernelEx) TJ_SYM(cuTensorMapEncodeTiled)
    TJ_SYM(cuGraphCreate) TJ_SYM(cuGraphAddKernelNode_v2) TJ_SYM_OPT(cuGraphAddDependencies_v2) TJ_SYM(cuGraphKernelNodeSetAttribute)
    TJ_SYM(cuGraphInstantiateWithFlags) TJ_SYM(cuGraphLaunch) TJ_SYM(cuGraphExecKernelNodeSetParams_v2)
    TJ_SYM(cuGraphExecDestroy) TJ_SYM(cuGraphDestroy) TJ_SYM(cuGetErrorString) TJ_SYM(cuEventCreate)
    TJ_SYM(cuEventDestroy_v2) TJ_SYM(cuEventRecord) TJ_SYM(cuEventSynchronize) TJ_SYM(cuEventElapsedTime)
    TJ_SYM_OPT(cuOccupancyMaxActiveClusters) TJ_SYM_OPT(cuMemGetAddressRange_v2) TJ_SYM_OPT(cuIpcGetMemHandle)
    TJ_SYM_OPT(cuIpcOpenMemHandle_v2) TJ_SYM_OPT(cuIpcCloseMemHandle)
#undef TJ_SYM
#undef TJ_SYM_OPT
    if (!all) return;
    CUresult r = cuInit(0);
    if (r != CUDA_SUCCESS) {
      why = "cuInit failed with code " + std::to_string(static_cast<int>(r));
      return;
    }
    ok = true;
  }
};

Driver& drv() {
  static Driver d;
  static std::once_flag once;
  std::call_once(once, [] { d.load(); });
  return d;
}

int cu_fail(CUresult r, const char* what) {
  const char* s = nullptr;
  if (drv().cuGetErrorString) drv().cuGetErrorString(r, &s);
  return fail(TJ_ERR_CUDA, "%s failed: CUDA error %d (%s)", what, static_cast<int>(r), s ? s : "?");
}

#define TJ_CU(call, what)                         \
  do {                                            \
    CUresult _r = (call);                         \
    if (_r != CUDA_SUCCESS) return cu_fail(_r, what); \
  } while (0)

struct CtxGuard {
  bool pushed = false;
  explicit CtxGuard(CUcontext c) {
    if (c && drv().cuCtxPushCurrent_v2(c) == CUDA_SUCCESS) pushed = true;
  }
  ~CtxGuard() {
    if (pushed) {
      CUcontext dummy;
      drv().cuCtxPopCurrent_v2(&dummy);
    }
  }
};

struct KernelRec {
  tj_launch launch{};
  std::string symbol;
  CUfunction fn = nullptr;
  std::vector<tj_argref> args;
  std::vector<tj_tmap> tmaps;
  // parameter block of the last launch (or of the graph node); 64-byte aligned storage
  std::vector<uint64_t> params;
  bool skip = false;
  CUgraphNode node = nullptr;
};

struct Program {
  int device = 0;
  CUcontext ctx = nullptr;
  std::vector<CUmodule> modules;
  std::vector<KernelRec> kernels;
  CUdeviceptr arena = 0;
  uint64_t arena_bytes = 0;
  CUdeviceptr status = 0;  // int32[4]: code, where, spare, spare
  int32_t num_inputs = 0, num_outputs = 0;
  bool graph_enabled = false;
  // programmatic dependent launch between the program's kernels: each kernel may start (set-up
  // only; it waits in griddepcontrol.wait) while the previous one finishes
  bool pdl = true;
  CUgraph graph = nullptr;
  CUgraphExec exec = nullptr;
  uint64_t calls = 0, launches = 0, replays = 0, node_updates = 0, instantiations = 0;
  std::string graph_label;  // NVTX range around a graph replay: "tj_b200 graph: <first> .. <last>"
  double host_us = 0.0;
  std::mutex mu;

  ~Program() {
    if (!drv().ok) return;
    CtxGuard g(ctx);
    if (exec) drv().cuGraphExecDestroy(exec);
    if (graph) drv().cuGraphDestroy(graph);
    if (arena) drv().cuMemFree_v2(arena);
    if (status) drv().cuMemFree_v2(status);
    for (CUmodule m : modules) drv().cuModuleUnload(m);
    if (ctx) {
      CUdevice dev;
      if (drv().cuDeviceGet(&dev, device) == CUDA_SUCCESS) drv().cuDevicePrimaryCtxRelease_v2(dev);
    }
  }
};

uint64_t resolve(const Program& p, const tj_argref& a, const void* const* in, void* const* out) {
  switch (a.kind) {
    case TJ_ARG_INPUT: return reinterpret_cast<uint64_t>(in[a.value]);
    case TJ_ARG_OUTPUT: return reinterpret_cast<uint64_t>(out[a.value]);
    case TJ_ARG_ARENA: return static_cast<uint64_t>(p.arena) + static_cast<uint64_t>(a.value);
    default: return static_cast<uint64_t>(p.status);
  }
}

// Fill k.params for this call; returns TJ_OK and sets *changed if the block differs.
int build_params(const Program& p, KernelRec& k, const void* const* in, void* const* out, bool* changed) {
  const size_t words = (k.launch.param_bytes + 7) / 8;
  uint64_t tmp_stack[512];
  std::vector<uint64_t> tmp_heap;
  uint64_t* tmp = tmp_stack;
  if (words > 512) {
    tmp_heap.assign(words, 0);
    tmp = tmp_heap.data();
  } else {
    std::memset(tmp, 0, words * 8);
  }
  for (size_t i = 0; i < k.args.size(); ++i) tmp[i] = resolve(p, k.args[i], in, out);
  for (const tj_tmap& t : k.tmaps) {
    alignas(64) CUtensorMap map;
    void* base = reinterpret_cast<void*>(tmp[t.arg]);
    cuuint64_t dims[5];
    cuuint64_t strides[4];
    cuuint32_t box[5], estr[5];
    for (int d = 0; d < t.rank; ++d) {
      dims[d] = t.dims[d];
      box[d] = t.box[d];
      estr[d] = 1;
    }
    for (int d = 0; d + 1 < t.rank; ++d) strides[d] = t.strides[d];
    CUresult r = drv().cuTensorMapEncodeTiled(
        &map, static_cast<CUtensorMapDataType>(t.dtype), static_cast<cuuint32_t>(t.rank), base, dims, strides, box,
        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, static_cast<CUtensorMapSwizzle>(t.swizzle),
        static_cast<CUtensorMapL2promotion>(t.l2_promotion), CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      return fail(TJ_ERR_CUDA, "cuTensorMapEncodeTiled for %s (arg %d, base %p, rank %d) failed with %d",
                  k.symbol.c_str(), t.arg, base, t.rank, static_cast<int>(r));
    }
    std::memcpy(reinterpret_cast<char*>(tmp) + t.param_offset, &map, sizeof(map));
  }
  *changed = k.params.size() != words || std::memcmp(k.params.data(), tmp, words * 8) != 0;
  if (*changed) {
    k.params.assign(tmp, tmp + words);
  }
  return TJ_OK;
}

int launch_direct(Program& p, KernelRec& k, CUstream s, bool pdl = false) {
  CUlaunchConfig cfg{};
  cfg.gridDimX = k.launch.grid[0];
  cfg.gridDimY = k.launch.grid[1];
  cfg.gridDimZ = k.launch.grid[2];
  cfg.blockDimX = k.launch.block[0];
  cfg.blockDimY = k.launch.block[1];
  cfg.blockDimZ = k.launch.block[2];
  cfg.sharedMemBytes = k.launch.smem_bytes;
  cfg.hStream = s;
  CUlaunchAttribute attr[2];
  unsigned nattr = 0;
  const uint32_t* c = k.launch.cluster;
  if (c[0] * c[1] * c[2] > 1) {
    attr[nattr].id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
    attr[nattr].value.clusterDim.x = c[0] ? c[0] : 1;
    attr[nattr].value.clusterDim.y = c[1] ? c[1] : 1;
    attr[nattr].value.clusterDim.z = c[2] ? c[2] : 1;
    ++nattr;
  }
  if (pdl) {
    attr[nattr].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
    attr[nattr].value.programmaticStreamSerializationAllowed = 1;
    ++nattr;
  }
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  void* kp[1] = {k.params.data()};
  nvtxRangePushA(k.symbol.c_str());
  CUresult r = drv().cuLaunchKernelEx(&cfg, k.fn, kp, nullptr);
  nvtxRangePop();
  if (r != CUDA_SUCCESS) return cu_fail(r, ("cuLaunchKernelEx " + k.symbol).c_str());
  p.launches++;
  return TJ_OK;
}

CUDA_KERNEL_NODE_PARAMS node_params(KernelRec& k, void** kp) {
  CUDA_KERNEL_NODE_PARAMS np{};
  np.func = k.fn;
  np.gridDimX = k.launch.grid[0];
  np.gridDimY = k.launch.grid[1];
  np.gridDimZ = k.launch.grid[2];
  np.blockDimX = k.launch.block[0];
  np.blockDimY = k.launch.block[1];
  np.blockDimZ = k.launch.block[2];
  np.sharedMemBytes = k.launch.smem_bytes;
  np.kernelParams = kp;
  np.extra = nullptr;
  return np;
}

int build_graph(Program& p) {
  TJ_CU(drv().cuGraphCreate(&p.graph, 0), "cuGraphCreate");
  CUgraphNode prev = nullptr;
  // consecutive kernels are joined by programmatic edges (the successor may start once every
  // block of the predecessor has triggered launch_dependents, and waits in griddepcontrol.wait
  // for its completion); plain edges when that is off or the driver lacks the call
  const bool pdl = p.pdl && drv().cuGraphAddDependencies_v2 != nullptr;
  for (KernelRec& k : p.kernels) {
    if (k.skip) continue;
    void* kp[1] = {k.params.data()};
    CUDA_KERNEL_NODE_PARAMS np = node_params(k, kp);
    const bool plain = prev && !pdl;
    TJ_CU(drv().cuGraphAddKernelNode_v2(&k.node, p.graph, plain ? &prev : nullptr, plain ? 1 : 0, &np),
          "cuGraphAddKernelNode");
    if (prev && pdl) {
      CUgraphEdgeData e{};
      e.from_port = CU_GRAPH_KERNEL_NODE_PORT_PROGRAMMATIC;
      e.to_port = 0;
      e.type = CU_GRAPH_DEPENDENCY_TYPE_PROGRAMMATIC;
      TJ_CU(drv().cuGraphAddDependencies_v2(p.graph, &prev, &k.node, &e, 1), "cuGraphAddDependencies");
    }
    const uint32_t* c = k.launch.cluster;
    if (c[0] * c[1] * c[2] > 1) {
      CUkernelNodeAttrValue v{};
      v.clusterDim.x = c[0];
      v.clusterDim.y = c[1] ? c[1] : 1;
      v.clusterDim.z = c[2] ? c[2] : 1;
      TJ_CU(drv().cuGraphKernelNodeSetAttribute(k.node, CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION, &v),
            "cuGraphKernelNodeSetAttribute(cluster)");
    }
    prev = k.node;
  }
  TJ_CU(drv().cuGraphInstantiateWithFlags(&p.exec, p.graph, 0), "cuGraphInstantiate");
  p.instantiations++;
  return TJ_OK;
}

}  // namespace

// Lets the other translation units of this library report through tj_b200_last_error().
void tj_b200_internal_set_error(const char* msg) { g_last_error = msg ? msg : ""; }

extern "C" {

int tj_b200_abi_version(void) { return TJ_B200_ABI_VERSION; }

const char* tj_b200_last_error(void) { return g_last_error.c_str(); }

int tj_b200_driver_available(void) {
  if (!drv().ok) return 0;
  int n = 0;
  if (drv().cuDeviceGetCount(&n) != CUDA_SUCCESS) return 0;
  return n > 0 ? 1 : 0;
}

int tj_b200_program_create(const void* const* cubins, const size_t* cubin_sizes, int32_t num_modules,
                           const tj_launch* launches, int32_t num_kernels, const tj_argref* args,
                           int32_t num_args_total, const tj_tmap* tmaps, int32_t num_tmaps_total,
                           uint64_t arena_bytes, int32_t num_inputs, int32_t num_outputs, int32_t device,
                           void** out_program) {
  if (!out_program) return fail(TJ_ERR_INVALID, "out_program is NULL");
  *out_program = nullptr;
  if (num_modules < 0 || num_kernels < 0 || num_args_total < 0 || num_tmaps_total < 0 || num_inputs < 0 ||
      num_outputs < 0)
    return fail(TJ_ERR_INVALID, "negative count");
  if ((num_modules && (!cubins || !cubin_sizes)) || (num_kernels && !launches) || (num_args_total && !args) ||
      (num_tmaps_total && !tmaps))
    return fail(TJ_ERR_INVALID, "NULL array with a non-zero count");
  // validate launches and argument references before touching the driver
  for (int32_t i = 0; i < num_kernels; ++i) {
    const tj_launch& L = launches[i];
    if (!L.symbol) return fail(TJ_ERR_INVALID, "kernel %d: NULL symbol", i);
    if (L.module < 0 || L.module >= num_modules) return fail(TJ_ERR_INVALID, "kernel %d: module out of range", i);
    if (L.first_arg < 0 || L.num_args < 0 || L.first_arg + L.num_args > num_args_total)
      return fail(TJ_ERR_INVALID, "kernel %d: argument slice out of range", i);
    if (L.first_tmap < 0 || L.num_tmaps < 0 || L.first_tmap + L.num_tmaps > num_tmaps_total)
      return fail(TJ_ERR_INVALID, "kernel %d: tensor-map slice out of range", i);
    if (static_cast<uint64_t>(L.num_args) * 8 > L.param_bytes)
      return fail(TJ_ERR_INVALID, "kernel %d: parameter block too small for its pointers", i);
    if (L.block[0] * L.block[1] * L.block[2] == 0 || L.block[0] * L.block[1] * L.block[2] > 1024)
      return fail(TJ_ERR_INVALID, "kernel %d: bad block size", i);
    for (int32_t j = 0; j < L.num_args; ++j) {
      const tj_argref& a = args[L.first_arg + j];
      switch (a.kind) {
        case TJ_ARG_INPUT:
          if (a.value < 0 || a.value >= num_inputs) return fail(TJ_ERR_INVALID, "kernel %d arg %d: input index out of range", i, j);
          break;
        case TJ_ARG_OUTPUT:
          if (a.value < 0 || a.value >= num_outputs) return fail(TJ_ERR_INVALID, "kernel %d arg %d: output index out of range", i, j);
          break;
        case TJ_ARG_ARENA:
          if (a.value < 0 || static_cast<uint64_t>(a.value) >= (arena_bytes ? arena_bytes : 1))
            return fail(TJ_ERR_INVALID, "kernel %d arg %d: arena offset out of range", i, j);
          break;
        case TJ_ARG_STATUS:
          break;
        default:
          return fail(TJ_ERR_INVALID, "kernel %d arg %d: bad argument kind %d", i, j, a.kind);
      }
    }
    for (int32_t j = 0; j < L.num_tmaps; ++j) {
      const tj_tmap& t = tmaps[L.first_tmap + j];
      if (t.arg < 0 || t.arg >= L.num_args) return fail(TJ_ERR_INVALID, "kernel %d tmap %d: arg out of range", i, j);
      if (t.rank < 1 || t.rank > 5) return fail(TJ_ERR_INVALID, "kernel %d tmap %d: bad rank", i, j);
      if (t.param_offset % 64 != 0 || t.param_offset + sizeof(CUtensorMap) > L.param_bytes ||
          t.param_offset < static_cast<uint32_t>(L.num_args) * 8)
        return fail(TJ_ERR_INVALID, "kernel %d tmap %d: bad parameter offset", i, j);
    }
  }
  Driver& d = drv();
  if (!d.ok) return fail(TJ_ERR_NO_DRIVER, "%s", d.why.c_str());

  std::unique_ptr<Program> p(new Program());
  p->device = device;
  p->num_inputs = num_inputs;
  p->num_outputs = num_outputs;
  CUdevice dev;
  TJ_CU(d.cuDeviceGet(&dev, device), "cuDeviceGet");
  TJ_CU(d.cuDevicePrimaryCtxRetain(&p->ctx, dev), "cuDevicePrimaryCtxRetain");
  CtxGuard guard(p->ctx);
  for (int32_t m = 0; m < num_modules; ++m) {
    CUmodule mod;
    if (cubin_sizes[m] < 16) return fail(TJ_ERR_INVALID, "module %d: image too small (%zu bytes)", m, cubin_sizes[m]);
    CUresult r = d.cuModuleLoadData(&mod, cubins[m]);
    if (r != CUDA_SUCCESS) return cu_fail(r, "cuModuleLoadData");
    p->modules.push_back(mod);
  }
  p->kernels.resize(num_kernels);
  for (int32_t i = 0; i < num_kernels; ++i) {
    KernelRec& k = p->kernels[i];
    k.launch = launches[i];
    k.symbol = launches[i].symbol;
    k.launch.symbol = nullptr;
    k.args.assign(args + launches[i].first_arg, args + launches[i].first_arg + launches[i].num_args);
    k.tmaps.assign(tmaps + launches[i].first_tmap, tmaps + launches[i].first_tmap + launches[i].num_tmaps);
    k.skip = k.launch.grid[0] == 0 || k.launch.grid[1] == 0 || k.launch.grid[2] == 0;
    CUresult r = d.cuModuleGetFunction(&k.fn, p->modules[k.launch.module], k.symbol.c_str());
    if (r != CUDA_SUCCESS) return cu_fail(r, ("cuModuleGetFunction " + k.symbol).c_str());
    if (k.launch.smem_bytes > 48 * 1024)
      TJ_CU(d.cuFuncSetAttribute(k.fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, k.launch.smem_bytes),
            "cuFuncSetAttribute(max dynamic smem)");
    const uint32_t* cl = k.launch.cluster;
    const uint32_t csize = (cl[0] ? cl[0] : 1) * (cl[1] ? cl[1] : 1) * (cl[2] ? cl[2] : 1);
    if (csize > 1 && d.cuOccupancyMaxActiveClusters && !k.skip) {
      // Cluster launches are persistent kernels (tiles strided by gridDim): clamp the grid to
      // the clusters that can be resident at once, so no cluster waits for a second wave.
      CUlaunchConfig cfg{};
      cfg.gridDimX = k.launch.grid[0];
      cfg.gridDimY = k.launch.grid[1];
      cfg.gridDimZ = k.launch.grid[2];
      cfg.blockDimX = k.launch.block[0];
      cfg.blockDimY = k.launch.block[1];
      cfg.blockDimZ = k.launch.block[2];
      cfg.sharedMemBytes = k.launch.smem_bytes;
      CUlaunchAttribute attr{};
      attr.id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
      attr.value.clusterDim.x = cl[0] ? cl[0] : 1;
      attr.value.clusterDim.y = cl[1] ? cl[1] : 1;
      attr.value.clusterDim.z = cl[2] ? cl[2] : 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int nclusters = 0;
      if (d.cuOccupancyMaxActiveClusters(&nclusters, k.fn, &cfg) == CUDA_SUCCESS && nclusters > 0 &&
          k.launch.grid[1] == 1 && k.launch.grid[2] == 1) {
        const uint32_t cap = static_cast<uint32_t>(nclusters) * attr.value.clusterDim.x;
        if (k.launch.grid[0] > cap) k.launch.grid[0] = cap;
      }
    }
    const char* pc = std::getenv("TENSORJIT_B200_PARAM_CHECK");
    if (d.cuFuncGetParamInfo && !(pc && pc[0] == '0')) {
      size_t off = 0, sz = 0;
      if (d.cuFuncGetParamInfo(k.fn, 0, &off, &sz) == CUDA_SUCCESS && sz != k.launch.param_bytes)
        return fail(TJ_ERR_INVALID, "kernel %s: parameter block is %zu bytes in the cubin, %u in the launch table",
                    k.symbol.c_str(), sz, k.launch.param_bytes);
    }
  }
  if (arena_bytes) {
    TJ_CU(d.cuMemAlloc_v2(&p->arena, arena_bytes), "cuMemAlloc(arena)");
    p->arena_bytes = arena_bytes;
  }
  TJ_CU(d.cuMemAlloc_v2(&p->status, 16), "cuMemAlloc(status)");
  TJ_CU(d.cuMemsetD32_v2(p->status, 0, 4), "cuMemsetD32(status)");
  {
    const char* e = std::getenv("TENSORJIT_B200_PDL");  // "0": kernels strictly one after the other
    p->pdl = !(e && e[0] == '0');
  }
  if (!p->kernels.empty())
    p->graph_label = "tj_b200 graph: " + p->kernels.front().symbol +
                     (p->kernels.size() > 1 ? " .. " + p->kernels.back().symbol : std::string());
  *out_program = p.release();
  return TJ_OK;
}

int tj_b200_run(void* program, const void* const* inputs, void* const* outputs, void* stream) {
  if (!program) return fail(TJ_ERR_INVALID, "program is NULL");
  Program& p = *static_cast<Program*>(program);
  if ((p.num_inputs && !inputs) || (p.num_outputs && !outputs)) return fail(TJ_ERR_INVALID, "NULL input/output array");
  std::lock_guard<std::mutex> lock(p.mu);
  const auto t0 = std::chrono::steady_clock::now();
  CtxGuard guard(p.ctx);
  CUstream s = reinterpret_cast<CUstream>(stream);
  int rc = TJ_OK;
  if (!p.graph_enabled) {
    bool first = true;
    for (KernelRec& k : p.kernels) {
      if (k.skip) continue;
      bool changed = false;
      if ((rc = build_params(p, k, inputs, outputs, &changed)) != TJ_OK) return rc;
      if ((rc = launch_direct(p, k, s, p.pdl && !first)) != TJ_OK) return rc;
      first = false;
    }
  } else {
    bool any_changed = false;
    std::vector<char> changed(p.kernels.size(), 0);
    for (size_t i = 0; i < p.kernels.size(); ++i) {
      KernelRec& k = p.kernels[i];
      if (k.skip) continue;
      bool c = false;
      if ((rc = build_params(p, k, inputs, outputs, &c)) != TJ_OK) return rc;
      changed[i] = c;
      any_changed |= c;
    }
    if (!p.exec) {
      if ((rc = build_graph(p)) != TJ_OK) return rc;
    } else if (any_changed) {
      for (size_t i = 0; i < p.kernels.size(); ++i) {
        KernelRec& k = p.kernels[i];
        if (k.skip || !changed[i]) continue;
        void* kp[1] = {k.params.data()};
        CUDA_KERNEL_NODE_PARAMS np = node_params(k, kp);
        TJ_CU(drv().cuGraphExecKernelNodeSetParams_v2(p.exec, k.node, &np), "cuGraphExecKernelNodeSetParams");
        p.node_updates++;
      }
    }
    nvtxRangePushA(p.graph_label.c_str());   // the graph's kernel nodes carry the plan kernels' names
    const CUresult gr = drv().cuGraphLaunch(p.exec, s);
    nvtxRangePop();
    TJ_CU(gr, "cuGraphLaunch");
    p.replays++;
  }
  p.calls++;
  p.host_us += std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count();
  return TJ_OK;
}

int tj_b200_time_kernels(void* program, const void* const* inputs, void* const* outputs, void* stream, int32_t iters,
                         float* ms_per_kernel) {
  if (!program || !ms_per_kernel || iters < 1) return fail(TJ_ERR_INVALID, "bad arguments to tj_b200_time_kernels");
  Program& p = *static_cast<Program*>(program);
  if ((p.num_inputs && !inputs) || (p.num_outputs && !outputs)) return fail(TJ_ERR_INVALID, "NULL input/output array");
  std::lock_guard<std::mutex> lock(p.mu);
  CtxGuard guard(p.ctx);
  CUstream s = reinterpret_cast<CUstream>(stream);
  const size_t nk = p.kernels.size();
  std::vector<CUevent> ev(nk + 1, nullptr);
  int rc = TJ_OK;
  for (auto& e : ev) {
    CUresult r = drv().cuEventCreate(&e, CU_EVENT_DEFAULT);
    if (r != CUDA_SUCCESS) { rc = cu_fail(r, "cuEventCreate"); break; }
  }
  std::vector<double> acc(nk, 0.0);
  for (int32_t it = 0; it < iters && rc == TJ_OK; ++it) {
    for (size_t i = 0; i < nk && rc == TJ_OK; ++i) {
      KernelRec& k = p.kernels[i];
      CUresult r = drv().cuEventRecord(ev[i], s);
      if (r != CUDA_SUCCESS) { rc = cu_fail(r, "cuEventRecord"); break; }
      if (k.skip) continue;
      bool changed = false;
      if ((rc = build_params(p, k, inputs, outputs, &changed)) != TJ_OK) break;
      rc = launch_direct(p, k, s);
    }
    if (rc != TJ_OK) break;
    CUresult r = drv().cuEventRecord(ev[nk], s);
    if (r == CUDA_SUCCESS) r = drv().cuEventSynchronize(ev[nk]);
    if (r != CUDA_SUCCESS) { rc = cu_fail(r, "cuEventSynchronize"); break; }
    for (size_t i = 0; i < nk; ++i) {
      float ms = 0.f;
      r = drv().cuEventElapsedTime(&ms, ev[i], ev[i + 1]);
      if (r != CUDA_SUCCESS) { rc = cu_fail(r, "cuEventElapsedTime"); break; }
      acc[i] += ms;
    }
  }
  for (auto& e : ev)
    if (e) drv().cuEventDestroy_v2(e);
  if (rc != TJ_OK) return rc;
  for (size_t i = 0; i < nk; ++i) ms_per_kernel[i] = static_cast<float>(acc[i] / iters);
  return TJ_OK;
}

int tj_b200_set_graph(void* program, int32_t enable) {
  if (!program) return fail(TJ_ERR_INVALID, "program is NULL");
  Program& p = *static_cast<Program*>(program);
  std::lock_guard<std::mutex> lock(p.mu);
  p.graph_enabled = enable != 0;
  return TJ_OK;
}

int tj_b200_set_pdl(void* program, int32_t enable) {
  if (!program) return fail(TJ_ERR_INVALID, "program is NULL");
  Program& p = *static_cast<Program*>(program);
  std::lock_guard<std::mutex> lock(p.mu);
  const bool on = enable != 0;
  if (on == p.pdl) return TJ_OK;
  p.pdl = on;
  if (p.exec || p.graph) {  // rebuilt with (or without) programmatic edges at the next run
    CtxGuard guard(p.ctx);
    if (p.exec) drv().cuGraphExecDestroy(p.exec);
    if (p.graph) drv().cuGraphDestroy(p.graph);
    p.exec = nullptr;
    p.graph = nullptr;
  }
  return TJ_OK;
}

int tj_b200_check_status(void* program, int32_t* code, int32_t* where) {
  if (!program) return fail(TJ_ERR_INVALID, "program is NULL");
  Program& p = *static_cast<Program*>(program);
  std::lock_guard<std::mutex> lock(p.mu);
  CtxGuard guard(p.ctx);
  TJ_CU(drv().cuCtxSynchronize(), "cuCtxSynchronize");
  int32_t words[4] = {0, 0, 0, 0};
  TJ_CU(drv().cuMemcpyDtoH_v2(words, p.status, sizeof(words)), "cuMemcpyDtoH(status)");
  if (code) *code = words[0];
  if (where) *where = words[1];
  if (words[0] != 0) {
    TJ_CU(drv().cuMemsetD32_v2(p.status, 0, 4), "cuMemsetD32(status)");
    return fail(TJ_ERR_DEVICE_STATUS, "a kernel reported status %d at %d", words[0], words[1]);
  }
  return TJ_OK;
}

int tj_b200_program_info(void* program, tj_program_info* info) {
  if (!program || !info) return fail(TJ_ERR_INVALID, "NULL argument");
  Program& p = *static_cast<Program*>(program);
  std::lock_guard<std::mutex> lock(p.mu);
  info->arena = reinterpret_cast<void*>(p.arena);
  info->arena_bytes = p.arena_bytes;
  info->num_kernels = static_cast<int32_t>(p.kernels.size());
  info->num_inputs = p.num_inputs;
  info->num_outputs = p.num_outputs;
  info->graph_enabled = p.graph_enabled ? 1 : 0;
  info->calls = p.calls;
  info->launches = p.launches;
  info->graph_replays = p.replays;
  info->graph_node_updates = p.node_updates;
  info->graph_instantiations = p.instantiations;
  info->host_us_total = p.host_us;
  return TJ_OK;
}

int tj_b200_destroy(void* program) {
  if (!program) return TJ_OK;
  delete static_cast<Program*>(program);
  return TJ_OK;
}

// -- peer memory between the processes of a node ------------------------------
// The primary context of `device` stays retained while one of its IPC mappings is open, so the
// mapping outlives a caller that drops its own reference to the context first.
static int ipc_driver(Driver** out) {
  Driver& d = drv();
  if (!d.ok) return fail(TJ_ERR_NO_DRIVER, "%s", d.why.c_str());
  if (!d.cuMemGetAddressRange_v2 || !d.cuIpcGetMemHandle || !d.cuIpcOpenMemHandle_v2 || !d.cuIpcCloseMemHandle)
    return fail(TJ_ERR_NOT_SUPPORTED, "this driver exports no CUDA IPC entry points");
  *out = &d;
  return TJ_OK;
}

int tj_b200_ipc_export(const void* dptr, int32_t device, tj_ipc_handle* handle, uint64_t* offset) {
  if (!dptr || !handle || !offset) return fail(TJ_ERR_INVALID, "NULL argument to tj_b200_ipc_export");
  Driver* d = nullptr;
  int rc = ipc_driver(&d);
  if (rc != TJ_OK) return rc;
  CUdevice dev;
  CUcontext ctx;
  TJ_CU(d->cuDeviceGet(&dev, device), "cuDeviceGet");
  TJ_CU(d->cuDevicePrimaryCtxRetain(&ctx, dev), "cuDevicePrimaryCtxRetain");
  {
    CtxGuard guard(ctx);
    CUdeviceptr base = 0;
    size_t size = 0;
    CUresult r = d->cuMemGetAddressRange_v2(&base, &size, reinterpret_cast<CUdeviceptr>(dptr));
    if (r == CUDA_SUCCESS) {
      CUipcMemHandle h;
      r = d->cuIpcGetMemHandle(&h, base);
      if (r == CUDA_SUCCESS) {
        static_assert(sizeof(h) == sizeof(handle->bytes), "CUipcMemHandle is 64 bytes");
        std::memcpy(handle->bytes, &h, sizeof(h));
        *offset = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(dptr) - base);
      }
    }
    if (r != CUDA_SUCCESS) rc = cu_fail(r, "cuIpcGetMemHandle");
  }
  d->cuDevicePrimaryCtxRelease_v2(dev);
  return rc;
}

int tj_b200_ipc_open(const tj_ipc_handle* handle, uint64_t offset, int32_t device, void** dptr) {
  if (!handle || !dptr) return fail(TJ_ERR_INVALID, "NULL argument to tj_b200_ipc_open");
  *dptr = nullptr;
  Driver* d = nullptr;
  int rc = ipc_driver(&d);
  if (rc != TJ_OK) return rc;
  CUdevice dev;
  CUcontext ctx;
  TJ_CU(d->cuDeviceGet(&dev, device), "cuDeviceGet");
  TJ_CU(d->cuDevicePrimaryCtxRetain(&ctx, dev), "cuDevicePrimaryCtxRetain");
  CUresult r;
  CUdeviceptr base = 0;
  {
    CtxGuard guard(ctx);
    CUipcMemHandle h;
    std::memcpy(&h, handle->bytes, sizeof(h));
    r = d->cuIpcOpenMemHandle_v2(&base, h, CU_IPC_MEM_LAZY_ENABLE_PEER_ACCESS);
  }
  if (r != CUDA_SUCCESS) {
    d->cuDevicePrimaryCtxRelease_v2(dev);
    return cu_fail(r, "cuIpcOpenMemHandle");
  }
  *dptr = reinterpret_cast<void*>(base + offset);   // the context stays retained until close
  return TJ_OK;
}

int tj_b200_ipc_close(void* dptr, uint64_t offset, int32_t device) {
  if (!dptr) return fail(TJ_ERR_INVALID, "NULL address to tj_b200_ipc_close");
  Driver* d = nullptr;
  int rc = ipc_driver(&d);
  if (rc != TJ_OK) return rc;
  CUdevice dev;
  CUcontext ctx;
  TJ_CU(d->cuDeviceGet(&dev, device), "cuDeviceGet");
  TJ_CU(d->cuDevicePrimaryCtxRetain(&ctx, dev), "cuDevicePrimaryCtxRetain");
  CUresult r;
  {
    CtxGuard guard(ctx);
    r = d->cuIpcCloseMemHandle(reinterpret_cast<CUdeviceptr>(dptr) - offset);
  }
  d->cuDevicePrimaryCtxRelease_v2(dev);       // this call's retain
  if (r != CUDA_SUCCESS) return cu_fail(r, "cuIpcCloseMemHandle");
  d->cuDevicePrimaryCtxRelease_v2(dev);       // the one taken by tj_b200_ipc_open
  return TJ_OK;
}

}  // extern "C"
