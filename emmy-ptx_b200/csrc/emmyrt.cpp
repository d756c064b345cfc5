// libemmyrt.so -- local B200 launcher for Emmy Kernel IR kernels.
//
// Replaces the reference's remote runner (docs/API.md) with the CUDA driver
// API on the local GPU.  The driver and NCCL are dlopen'd on first use, so
// this library loads anywhere and reports EMMY_ENODRIVER / EMMY_ENONCCL as a
// status instead of failing at load time.
#include "emmyrt.h"

#include <cuda.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

namespace {

thread_local std::string g_err;

int fail(int code, const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

// ---------------------------------------------------------------------------
// driver API table
// ---------------------------------------------------------------------------
struct Driver {
  bool ok = false;
  std::string why;
#define EMMY_FN(name) decltype(&::name) name = nullptr;
  EMMY_FN(cuInit)
  EMMY_FN(cuDeviceGetCount)
  EMMY_FN(cuDeviceGet)
  EMMY_FN(cuDeviceGetAttribute)
  EMMY_FN(cuDeviceGetName)
  EMMY_FN(cuDeviceTotalMem)
  EMMY_FN(cuDevicePrimaryCtxRetain)
  EMMY_FN(cuDevicePrimaryCtxRelease)
  EMMY_FN(cuCtxSetCurrent)
  EMMY_FN(cuCtxSynchronize)
  EMMY_FN(cuModuleLoadDataEx)
  EMMY_FN(cuModuleUnload)
  EMMY_FN(cuModuleGetFunction)
  EMMY_FN(cuModuleGetGlobal)
  EMMY_FN(cuFuncGetAttribute)
  EMMY_FN(cuFuncSetAttribute)
  EMMY_FN(cuLaunchKernel)
  EMMY_FN(cuMemAlloc)
  EMMY_FN(cuMemFree)
  EMMY_FN(cuMemAllocHost)
  EMMY_FN(cuMemFreeHost)
  EMMY_FN(cuMemcpyHtoDAsync)
  EMMY_FN(cuMemcpyDtoHAsync)
  EMMY_FN(cuMemcpyDtoDAsync)
  EMMY_FN(cuMemsetD32Async)
  EMMY_FN(cuStreamCreate)
  EMMY_FN(cuStreamDestroy)
  EMMY_FN(cuStreamSynchronize)
  EMMY_FN(cuEventCreate)
  EMMY_FN(cuEventDestroy)
  EMMY_FN(cuEventRecord)
  EMMY_FN(cuEventSynchronize)
  EMMY_FN(cuEventElapsedTime)
  EMMY_FN(cuStreamWaitEvent)
  EMMY_FN(cuGetErrorString)
  EMMY_FN(cuTensorMapEncodeTiled)
  EMMY_FN(cuIpcGetMemHandle)
  EMMY_FN(cuIpcOpenMemHandle)
  EMMY_FN(cuIpcCloseMemHandle)
  EMMY_FN(cuLaunchKernelEx)  // optional: only launches that overlap their predecessor use it
#undef EMMY_FN
};

Driver g_drv;
std::once_flag g_drv_once;

void load_driver() {
  void *h = dlopen("libcuda.so.1", RTLD_NOW | RTLD_GLOBAL);
  if (!h) {
    g_drv.why = std::string("cannot load libcuda.so.1: ") + dlerror();
    return;
  }
  bool all = true;
  auto sym = [&](const char *n) {
    void *p = dlsym(h, n);
    if (!p) {
      all = false;
      g_drv.why = std::string("libcuda.so.1 lacks ") + n;
    }
    return p;
  };
#define EMMY_LOAD(field, name) g_drv.field = reinterpret_cast<decltype(g_drv.field)>(sym(name));
  EMMY_LOAD(cuInit, "cuInit")
  EMMY_LOAD(cuDeviceGetCount, "cuDeviceGetCount")
  EMMY_LOAD(cuDeviceGet, "cuDeviceGet")
  EMMY_LOAD(cuDeviceGetAttribute, "cuDeviceGetAttribute")
  EMMY_LOAD(cuDeviceGetName, "cuDeviceGetName")
  EMMY_LOAD(cuDeviceTotalMem, "cuDeviceTotalMem_v2")
  EMMY_LOAD(cuDevicePrimaryCtxRetain, "cuDevicePrimaryCtxRetain")
  EMMY_LOAD(cuDevicePrimaryCtxRelease, "cuDevicePrimaryCtxRelease_v2")
  EMMY_LOAD(cuCtxSetCurrent, "cuCtxSetCurrent")
  EMMY_LOAD(cuCtxSynchronize, "cuCtxSynchronize")
  EMMY_LOAD(cuModuleLoadDataEx, "cuModuleLoadDataEx")
  EMMY_LOAD(cuModuleUnload, "cuModuleUnload")
  EMMY_LOAD(cuModuleGetFunction, "cuModuleGetFunction")
  EMMY_LOAD(cuModuleGetGlobal, "cuModuleGetGlobal_v2")
  EMMY_LOAD(cuFuncGetAttribute, "cuFuncGetAttribute")
  EMMY_LOAD(cuFuncSetAttribute, "cuFuncSetAttribute")
  EMMY_LOAD(cuLaunchKernel, "cuLaunchKernel")
  EMMY_LOAD(cuMemAlloc, "cuMemAlloc_v2")
  EMMY_LOAD(cuMemFree, "cuMemFree_v2")
  EMMY_LOAD(cuMemAllocHost, "cuMemAllocHost_v2")
  EMMY_LOAD(cuMemFreeHost, "cuMemFreeHost")
  EMMY_LOAD(cuMemcpyHtoDAsync, "cuMemcpyHtoDAsync_v2")
  EMMY_LOAD(cuMemcpyDtoHAsync, "cuMemcpyDtoHAsync_v2")
  EMMY_LOAD(cuMemcpyDtoDAsync, "cuMemcpyDtoDAsync_v2")
  EMMY_LOAD(cuMemsetD32Async, "cuMemsetD32Async")
  EMMY_LOAD(cuStreamCreate, "cuStreamCreate")
  EMMY_LOAD(cuStreamDestroy, "cuStreamDestroy_v2")
  EMMY_LOAD(cuStreamSynchronize, "cuStreamSynchronize")
  EMMY_LOAD(cuEventCreate, "cuEventCreate")
  EMMY_LOAD(cuEventDestroy, "cuEventDestroy_v2")
  EMMY_LOAD(cuEventRecord, "cuEventRecord")
  EMMY_LOAD(cuEventSynchronize, "cuEventSynchronize")
  EMMY_LOAD(cuEventElapsedTime, "cuEventElapsedTime")
  EMMY_LOAD(cuStreamWaitEvent, "cuStreamWaitEvent")
  EMMY_LOAD(cuGetErrorString, "cuGetErrorString")
  EMMY_LOAD(cuTensorMapEncodeTiled, "cuTensorMapEncodeTiled")
  EMMY_LOAD(cuIpcGetMemHandle, "cuIpcGetMemHandle")
  EMMY_LOAD(cuIpcOpenMemHandle, "cuIpcOpenMemHandle_v2")
  EMMY_LOAD(cuIpcCloseMemHandle, "cuIpcCloseMemHandle")
#undef EMMY_LOAD
  g_drv.cuLaunchKernelEx =
      reinterpret_cast<decltype(g_drv.cuLaunchKernelEx)>(dlsym(h, "cuLaunchKernelEx"));
  if (!all) return;
  CUresult r = g_drv.cuInit(0);
  if (r != CUDA_SUCCESS) {
    g_drv.why = "cuInit failed with CUresult " + std::to_string(int(r));
    return;
  }
  g_drv.ok = true;
}

bool driver() {
  std::call_once(g_drv_once, load_driver);
  if (!g_drv.ok) fail(EMMY_ENODRIVER, "%s", g_drv.why.c_str());
  return g_drv.ok;
}

int cu(CUresult r, const char *what) {
  if (r == CUDA_SUCCESS) return EMMY_OK;
  const char *s = nullptr;
  if (g_drv.cuGetErrorString) g_drv.cuGetErrorString(r, &s);
  return fail(int(r), "%s: %s (CUresult %d)", what, s ? s : "unknown error", int(r));
}

#define DRV_OR_FAIL() \
  do {                \
    if (!driver()) return EMMY_ENODRIVER; \
  } while (0)

#define CU_TRY(call, what)                \
  do {                                    \
    int _rc = cu((call), (what));         \
    if (_rc != EMMY_OK) return _rc;       \
  } while (0)

// ---------------------------------------------------------------------------
// NCCL table
// ---------------------------------------------------------------------------
struct Nccl {
  bool ok = false;
  std::string why;
  decltype(&::ncclGetUniqueId) GetUniqueId = nullptr;
  decltype(&::ncclCommInitRank) CommInitRank = nullptr;
  decltype(&::ncclAllReduce) AllReduce = nullptr;
  decltype(&::ncclCommDestroy) CommDestroy = nullptr;
  decltype(&::ncclCommAbort) CommAbort = nullptr;
  decltype(&::ncclCommGetAsyncError) CommGetAsyncError = nullptr;
  decltype(&::ncclGetErrorString) GetErrorString = nullptr;
};
Nccl g_nccl;
std::once_flag g_nccl_once;

void load_nccl() {
  void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) {
    g_nccl.why = std::string("cannot load libnccl.so.2: ") + dlerror();
    return;
  }
  bool all = true;
  auto sym = [&](const char *n) {
    void *p = dlsym(h, n);
    if (!p) {
      all = false;
      g_nccl.why = std::string("libnccl.so.2 lacks ") + n;
    }
    return p;
  };
  g_nccl.GetUniqueId = reinterpret_cast<decltype(g_nccl.GetUniqueId)>(sym("ncclGetUniqueId"));
  g_nccl.CommInitRank = reinterpret_cast<decltype(g_nccl.CommInitRank)>(sym("ncclCommInitRank"));
  g_nccl.AllReduce = reinterpret_cast<decltype(g_nccl.AllReduce)>(sym("ncclAllReduce"));
  g_nccl.CommDestroy = reinterpret_cast<decltype(g_nccl.CommDestroy)>(sym("ncclCommDestroy"));
  g_nccl.CommAbort = reinterpret_cast<decltype(g_nccl.CommAbort)>(sym("ncclCommAbort"));
  g_nccl.CommGetAsyncError =
      reinterpret_cast<decltype(g_nccl.CommGetAsyncError)>(sym("ncclCommGetAsyncError"));
  g_nccl.GetErrorString =
      reinterpret_cast<decltype(g_nccl.GetErrorString)>(sym("ncclGetErrorString"));
  g_nccl.ok = all;
}

bool nccl() {
  std::call_once(g_nccl_once, load_nccl);
  if (!g_nccl.ok) fail(EMMY_ENONCCL, "%s", g_nccl.why.c_str());
  return g_nccl.ok;
}

int nc(ncclResult_t r, const char *what) {
  if (r == ncclSuccess) return EMMY_OK;
  const char *s = g_nccl.GetErrorString ? g_nccl.GetErrorString(r) : "unknown";
  return fail(int(r), "%s: %s (ncclResult %d)", what, s, int(r));
}

}  // namespace

// ---------------------------------------------------------------------------
// objects
// ---------------------------------------------------------------------------
struct emmy_ctx {
  CUdevice dev;
  CUcontext cu;
  int ordinal;
};

struct emmy_mod {
  emmy_ctx *ctx;
  CUmodule mod;
  std::unordered_map<std::string, CUfunction> funcs;
  std::unordered_map<std::string, int> smem_set;  // max dynamic smem already granted
};

struct emmy_comm {
  ncclComm_t comm;
};

// Lets other translation units of this library set the message
// emmy_last_error() returns; hidden, so it is not part of the C ABI.
__attribute__((visibility("hidden"))) void emmyrt_set_last_error(const char *msg) { g_err = msg; }

extern "C" {

const char *emmy_version(void) { return "emmyrt 1.0 (sm_100a)"; }
const char *emmy_last_error(void) { return g_err.c_str(); }

int emmy_device_count(int *count) {
  if (!count) return fail(EMMY_EINVAL, "null count");
  DRV_OR_FAIL();
  CU_TRY(g_drv.cuDeviceGetCount(count), "cuDeviceGetCount");
  return EMMY_OK;
}

int emmy_ctx_create(int device, emmy_ctx **out) {
  if (!out) return fail(EMMY_EINVAL, "null out");
  DRV_OR_FAIL();
  auto *c = new emmy_ctx();
  c->ordinal = device;
  int rc = cu(g_drv.cuDeviceGet(&c->dev, device), "cuDeviceGet");
  if (rc == EMMY_OK) rc = cu(g_drv.cuDevicePrimaryCtxRetain(&c->cu, c->dev), "cuDevicePrimaryCtxRetain");
  if (rc == EMMY_OK) rc = cu(g_drv.cuCtxSetCurrent(c->cu), "cuCtxSetCurrent");
  if (rc != EMMY_OK) {
    delete c;
    return rc;
  }
  *out = c;
  return EMMY_OK;
}

int emmy_ctx_destroy(emmy_ctx *ctx) {
  if (!ctx) return EMMY_OK;
  DRV_OR_FAIL();
  int rc = cu(g_drv.cuDevicePrimaryCtxRelease(ctx->dev), "cuDevicePrimaryCtxRelease");
  delete ctx;
  return rc;
}

int emmy_ctx_make_current(emmy_ctx *ctx) {
  if (!ctx) return fail(EMMY_EINVAL, "null ctx");
  DRV_OR_FAIL();
  CU_TRY(g_drv.cuCtxSetCurrent(ctx->cu), "cuCtxSetCurrent");
  return EMMY_OK;
}

int emmy_ctx_synchronize(emmy_ctx *ctx) {
  DRV_OR_FAIL();
  if (ctx) CU_TRY(g_drv.cuCtxSetCurrent(ctx->cu), "cuCtxSetCurrent");
  CU_TRY(g_drv.cuCtxSynchronize(), "cuCtxSynchronize");
  return EMMY_OK;
}

int emmy_device_info(emmy_ctx *ctx, int *sm_count, int *cc_major, int *cc_minor,
                     size_t *total_mem, char *name, int name_len) {
  if (!ctx) return fail(EMMY_EINVAL, "null ctx");
  DRV_OR_FAIL();
  if (sm_count)
    CU_TRY(g_drv.cuDeviceGetAttribute(sm_count, CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT, ctx->dev),
           "cuDeviceGetAttribute");
  if (cc_major)
    CU_TRY(g_drv.cuDeviceGetAttribute(cc_major, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MAJOR, ctx->dev),
           "cuDeviceGetAttribute");
  if (cc_minor)
    CU_TRY(g_drv.cuDeviceGetAttribute(cc_minor, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MINOR, ctx->dev),
           "cuDeviceGetAttribute");
  if (total_mem) CU_TRY(g_drv.cuDeviceTotalMem(total_mem, ctx->dev), "cuDeviceTotalMem");
  if (name && name_len > 0) CU_TRY(g_drv.cuDeviceGetName(name, name_len, ctx->dev), "cuDeviceGetName");
  return EMMY_OK;
}

int emmy_module_load(emmy_ctx *ctx, const char *ptx, emmy_mod **out, char *log, size_t log_len) {
  if (!ctx || !ptx || !out) return fail(EMMY_EINVAL, "null argument");
  DRV_OR_FAIL();
  CU_TRY(g_drv.cuCtxSetCurrent(ctx->cu), "cuCtxSetCurrent");
  static char errbuf[16384];
  errbuf[0] = 0;
  CUjit_option opts[2] = {CU_JIT_ERROR_LOG_BUFFER, CU_JIT_ERROR_LOG_BUFFER_SIZE_BYTES};
  void *vals[2] = {errbuf, reinterpret_cast<void *>(static_cast<uintptr_t>(sizeof errbuf))};
  CUmodule m;
  CUresult r = g_drv.cuModuleLoadDataEx(&m, ptx, 2, opts, vals);
  if (log && log_len) {
    strncpy(log, errbuf, log_len - 1);
    log[log_len - 1] = 0;
  }
  if (r != CUDA_SUCCESS) {
    int rc = cu(r, "cuModuleLoadDataEx");
    g_err += std::string(": ") + errbuf;
    return rc;
  }
  auto *mod = new emmy_mod();
  mod->ctx = ctx;
  mod->mod = m;
  *out = mod;
  return EMMY_OK;
}

int emmy_module_unload(emmy_mod *mod) {
  if (!mod) return EMMY_OK;
  DRV_OR_FAIL();
  g_drv.cuCtxSetCurrent(mod->ctx->cu);
  int rc = cu(g_drv.cuModuleUnload(mod->mod), "cuModuleUnload");
  delete mod;
  return rc;
}

int emmy_module_global(emmy_mod *mod, const char *sym, emmy_dptr *ptr, size_t *bytes) {
  if (!mod || !sym) return fail(EMMY_EINVAL, "null argument");
  DRV_OR_FAIL();
  CUdeviceptr p = 0;
  size_t n = 0;
  CUresult r = g_drv.cuModuleGetGlobal(&p, &n, mod->mod, sym);
  if (r == CUDA_ERROR_NOT_FOUND) return fail(EMMY_ESYMBOL, "module has no global %s", sym);
  CU_TRY(r, "cuModuleGetGlobal");
  if (ptr) *ptr = p;
  if (bytes) *bytes = n;
  return EMMY_OK;
}

static int get_func(emmy_mod *mod, const char *entry, CUfunction *f) {
  auto it = mod->funcs.find(entry);
  if (it != mod->funcs.end()) {
    *f = it->second;
    return EMMY_OK;
  }
  CUresult r = g_drv.cuModuleGetFunction(f, mod->mod, entry);
  if (r == CUDA_ERROR_NOT_FOUND) return fail(EMMY_ENOENTRY, "no entry point %s in module", entry);
  CU_TRY(r, "cuModuleGetFunction");
  mod->funcs[entry] = *f;
  return EMMY_OK;
}

int emmy_func_info(emmy_mod *mod, const char *entry, int *regs, int *static_smem,
                   int *max_threads, int *local_bytes) {
  if (!mod || !entry) return fail(EMMY_EINVAL, "null argument");
  DRV_OR_FAIL();
  CUfunction f;
  int rc = get_func(mod, entry, &f);
  if (rc) return rc;
  if (regs) CU_TRY(g_drv.cuFuncGetAttribute(regs, CU_FUNC_ATTRIBUTE_NUM_REGS, f), "cuFuncGetAttribute");
  if (static_smem)
    CU_TRY(g_drv.cuFuncGetAttribute(static_smem, CU_FUNC_ATTRIBUTE_SHARED_SIZE_BYTES, f),
           "cuFuncGetAttribute");
  if (max_threads)
    CU_TRY(g_drv.cuFuncGetAttribute(max_threads, CU_FUNC_ATTRIBUTE_MAX_THREADS_PER_BLOCK, f),
           "cuFuncGetAttribute");
  if (local_bytes)
    CU_TRY(g_drv.cuFuncGetAttribute(local_bytes, CU_FUNC_ATTRIBUTE_LOCAL_SIZE_BYTES, f),
           "cuFuncGetAttribute");
  return EMMY_OK;
}

int emmy_launch(emmy_mod *mod, const char *entry, const uint32_t grid[3], const uint32_t block[3],
                uint32_t smem_bytes, void **args, emmy_stream stream) {
  if (!mod || !entry || !grid || !block) return fail(EMMY_EINVAL, "null argument");
  DRV_OR_FAIL();
  CUfunction f;
  int rc = get_func(mod, entry, &f);
  if (rc) return rc;
  if (smem_bytes > 48 * 1024) {
    auto it = mod->smem_set.find(entry);
    if (it == mod->smem_set.end() || it->second < int(smem_bytes)) {
      CU_TRY(g_drv.cuFuncSetAttribute(f, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                      int(smem_bytes)),
             "cuFuncSetAttribute(max dynamic smem)");
      mod->smem_set[entry] = int(smem_bytes);
    }
  }
  CU_TRY(g_drv.cuLaunchKernel(f, grid[0], grid[1], grid[2], block[0], block[1], block[2],
                              smem_bytes, static_cast<CUstream>(stream), args, nullptr),
         "cuLaunchKernel");
  return EMMY_OK;
}

int emmy_launch_ex(emmy_mod *mod, const char *entry, const uint32_t grid[3],
                   const uint32_t block[3], uint32_t smem_bytes, void **args, emmy_stream stream,
                   uint32_t flags) {
  if ((flags & ~uint32_t(EMMY_LAUNCH_OVERLAP_PREV)) != 0)
    return fail(EMMY_EINVAL, "unknown launch flags 0x%x", flags);
  if (!(flags & EMMY_LAUNCH_OVERLAP_PREV))
    return emmy_launch(mod, entry, grid, block, smem_bytes, args, stream);
  if (!mod || !entry || !grid || !block) return fail(EMMY_EINVAL, "null argument");
  DRV_OR_FAIL();
  if (!g_drv.cuLaunchKernelEx) return fail(EMMY_ENODRIVER, "libcuda.so.1 lacks cuLaunchKernelEx");
  CUfunction f;
  int rc = get_func(mod, entry, &f);
  if (rc) return rc;
  if (smem_bytes > 48 * 1024) {
    auto it = mod->smem_set.find(entry);
    if (it == mod->smem_set.end() || it->second < int(smem_bytes)) {
      CU_TRY(g_drv.cuFuncSetAttribute(f, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                      int(smem_bytes)),
             "cuFuncSetAttribute(max dynamic smem)");
      mod->smem_set[entry] = int(smem_bytes);
    }
  }
  // programmatic stream serialization: this grid may be scheduled once the
  // previous kernel in the stream has triggered (griddepcontrol.launch_
  // dependents) instead of once it has completed; the kernel itself waits
  // (griddepcontrol.wait) before its first write
  CUlaunchAttribute attr[1];
  memset(attr, 0, sizeof attr);
  attr[0].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
  attr[0].value.programmaticStreamSerializationAllowed = 1;
  CUlaunchConfig cfg;
  memset(&cfg, 0, sizeof cfg);
  cfg.gridDimX = grid[0];
  cfg.gridDimY = grid[1];
  cfg.gridDimZ = grid[2];
  cfg.blockDimX = block[0];
  cfg.blockDimY = block[1];
  cfg.blockDimZ = block[2];
  cfg.sharedMemBytes = smem_bytes;
  cfg.hStream = static_cast<CUstream>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CU_TRY(g_drv.cuLaunchKernelEx(&cfg, f, args, nullptr), "cuLaunchKernelEx");
  return EMMY_OK;
}

int emmy_launch_ptrs(emmy_mod *mod, const char *entry, const uint32_t grid[3],
                     const uint32_t block[3], uint32_t smem_bytes, const emmy_dptr *ptrs, int nptrs,
                     emmy_stream stream) {
  if (nptrs < 0 || nptrs > 64) return fail(EMMY_EINVAL, "bad parameter count %d", nptrs);
  emmy_dptr vals[64];
  void *args[64];
  for (int i = 0; i < nptrs; ++i) {
    vals[i] = ptrs[i];
    args[i] = &vals[i];
  }
  return emmy_launch(mod, entry, grid, block, smem_bytes, args, stream);
}

int emmy_tmap_encode(const emmy_tmap_desc *d, void *out128) {
  if (!d || !out128) return fail(EMMY_EINVAL, "null argument");
  if (d->rank < 1 || d->rank > 5) return fail(EMMY_EINVAL, "tensor map rank %u", d->rank);
  if (d->base % 16) return fail(EMMY_EINVAL, "tensor map base not 16-byte aligned");
  DRV_OR_FAIL();
  CUtensorMapDataType dt;
  switch (d->dtype) {
    case EMMY_TMAP_F32: dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32; break;
    case EMMY_TMAP_BF16: dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; break;
    case EMMY_TMAP_F16: dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; break;
    case EMMY_TMAP_U8: dt = CU_TENSOR_MAP_DATA_TYPE_UINT8; break;
    default: return fail(EMMY_EINVAL, "tensor map dtype %u", d->dtype);
  }
  CUtensorMapSwizzle sw;
  switch (d->swizzle) {
    case 0: sw = CU_TENSOR_MAP_SWIZZLE_NONE; break;
    case 32: sw = CU_TENSOR_MAP_SWIZZLE_32B; break;
    case 64: sw = CU_TENSOR_MAP_SWIZZLE_64B; break;
    case 128: sw = CU_TENSOR_MAP_SWIZZLE_128B; break;
    default: return fail(EMMY_EINVAL, "tensor map swizzle %u", d->swizzle);
  }
  CUtensorMapL2promotion l2;
  switch (d->l2_promote) {
    case 0: l2 = CU_TENSOR_MAP_L2_PROMOTION_NONE; break;
    case 64: l2 = CU_TENSOR_MAP_L2_PROMOTION_L2_64B; break;
    case 128: l2 = CU_TENSOR_MAP_L2_PROMOTION_L2_128B; break;
    default: l2 = CU_TENSOR_MAP_L2_PROMOTION_L2_256B; break;
  }
  cuuint64_t dims[5], strides[4];
  cuuint32_t box[5], estr[5];
  for (uint32_t i = 0; i < d->rank; ++i) {
    dims[i] = d->dims[i];
    box[i] = d->box[i];
    estr[i] = 1;
    if (i + 1 < d->rank) {
      if (d->strides[i] % 16) return fail(EMMY_EINVAL, "tensor map stride %u not 16-byte multiple", i);
      strides[i] = d->strides[i];
    }
  }
  CU_TRY(g_drv.cuTensorMapEncodeTiled(reinterpret_cast<CUtensorMap *>(out128), dt, d->rank,
                                      reinterpret_cast<void *>(d->base), dims, strides, box, estr,
                                      CU_TENSOR_MAP_INTERLEAVE_NONE, sw, l2,
                                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
         "cuTensorMapEncodeTiled");
  return EMMY_OK;
}

int emmy_tmap_fill(emmy_mod *mod, const char *sym, const emmy_tmap_desc *desc, emmy_stream stream) {
  alignas(64) unsigned char map[128];
  int rc = emmy_tmap_encode(desc, map);
  if (rc) return rc;
  emmy_dptr p = 0;
  size_t n = 0;
  rc = emmy_module_global(mod, sym, &p, &n);
  if (rc) return rc;
  if (n < 128) return fail(EMMY_EINVAL, "global %s is %zu bytes, a tensor map needs 128", sym, n);
  // Synchronous copy: the 128 bytes live on this stack frame.
  CU_TRY(g_drv.cuMemcpyHtoDAsync(p, map, 128, static_cast<CUstream>(stream)), "cuMemcpyHtoDAsync");
  CU_TRY(g_drv.cuStreamSynchronize(static_cast<CUstream>(stream)), "cuStreamSynchronize");
  return EMMY_OK;
}

int emmy_mem_alloc(emmy_ctx *ctx, size_t bytes, emmy_dptr *out) {
  if (!ctx || !out) return fail(EMMY_EINVAL, "null argument");
  DRV_OR_FAIL();
  CU_TRY(g_drv.cuCtxSetCurrent(ctx->cu), "cuCtxSetCurrent");
  CUdeviceptr p = 0;
  CU_TRY(g_drv.cuMemAlloc(&p, bytes ? bytes : 16), "cuMemAlloc");
  *out = p;
  return EMMY_OK;
}

int emmy_mem_free(emmy_ctx *ctx, emmy_dptr ptr) {
  DRV_OR_FAIL();
  if (ctx) g_drv.cuCtxSetCurrent(ctx->cu);
  CU_TRY(g_drv.cuMemFree(ptr), "cuMemFree");
  return EMMY_OK;
}

int emmy_host_alloc(emmy_ctx *ctx, size_t bytes, void **out) {
  if (!ctx || !out) return fail(EMMY_EINVAL, "null argument");
  DRV_OR_FAIL();
  CU_TRY(g_drv.cuCtxSetCurrent(ctx->cu), "cuCtxSetCurrent");
  CU_TRY(g_drv.cuMemAllocHost(out, bytes ? bytes : 16), "cuMemAllocHost");
  return EMMY_OK;
}

int emmy_host_free(emmy_ctx *ctx, void *ptr) {
  DRV_OR_FAIL();
  if (ctx) g_drv.cuCtxSetCurrent(ctx->cu);
  CU_TRY(g_drv.cuMemFreeHost(ptr), "cuMemFreeHost");
  return EMMY_OK;
}

int emmy_memcpy_htod(emmy_dptr dst, const void *src, size_t bytes, emmy_stream stream) {
  DRV_OR_FAIL();
  CU_TRY(g_drv.cuMemcpyHtoDAsync(dst, src, bytes, static_cast<CUstream>(stream)), "cuMemcpyHtoDAsync");
  return EMMY_OK;
}

int emmy_memcpy_dtoh(void *dst, emmy_dptr src, size_t bytes, emmy_stream stream) {
  DRV_OR_FAIL();
  CU_TRY(g_drv.cuMemcpyDtoHAsync(dst, src, bytes, static_cast<CUstream>(stream)), "cuMemcpyDtoHAsync");
  return EMMY_OK;
}

int emmy_memcpy_dtod(emmy_dptr dst, emmy_dptr src, size_t bytes, emmy_stream stream) {
  DRV_OR_FAIL();
  CU_TRY(g_drv.cuMemcpyDtoDAsync(dst, src, bytes, static_cast<CUstream>(stream)), "cuMemcpyDtoDAsync");
  return EMMY_OK;
}

int emmy_ipc_handle(emmy_ctx *ctx, emmy_dptr ptr, void *out64) {
  if (!ctx || !out64) return fail(EMMY_EINVAL, "null argument");
  DRV_OR_FAIL();
  CU_TRY(g_drv.cuCtxSetCurrent(ctx->cu), "cuCtxSetCurrent");
  CUipcMemHandle h;
  CU_TRY(g_drv.cuIpcGetMemHandle(&h, ptr), "cuIpcGetMemHandle");
  static_assert(sizeof(h) == 64, "CUipcMemHandle is 64 bytes");
  std::memcpy(out64, &h, sizeof(h));
  return EMMY_OK;
}

int emmy_ipc_open(emmy_ctx *ctx, const void *handle64, emmy_dptr *out) {
  if (!ctx || !handle64 || !out) return fail(EMMY_EINVAL, "null argument");
  DRV_OR_FAIL();
  CU_TRY(g_drv.cuCtxSetCurrent(ctx->cu), "cuCtxSetCurrent");
  CUipcMemHandle h;
  std::memcpy(&h, handle64, sizeof(h));
  CUdeviceptr p = 0;
  CU_TRY(g_drv.cuIpcOpenMemHandle(&p, h, CU_IPC_MEM_LAZY_ENABLE_PEER_ACCESS),
         "cuIpcOpenMemHandle");
  *out = p;
  return EMMY_OK;
}

int emmy_ipc_close(emmy_ctx *ctx, emmy_dptr ptr) {
  if (!ctx) return fail(EMMY_EINVAL, "null ctx");
  DRV_OR_FAIL();
  CU_TRY(g_drv.cuCtxSetCurrent(ctx->cu), "cuCtxSetCurrent");
  CU_TRY(g_drv.cuIpcCloseMemHandle(ptr), "cuIpcCloseMemHandle");
  return EMMY_OK;
}

int emmy_memset_d32(emmy_dptr dst, uint32_t value, size_t count, emmy_stream stream) {
  DRV_OR_FAIL();
  CU_TRY(g_drv.cuMemsetD32Async(dst, value, count, static_cast<CUstream>(stream)), "cuMemsetD32Async");
  return EMMY_OK;
}

int emmy_stream_create(emmy_ctx *ctx, emmy_stream *out) {
  if (!ctx || !out) return fail(EMMY_EINVAL, "null argument");
  DRV_OR_FAIL();
  CU_TRY(g_drv.cuCtxSetCurrent(ctx->cu), "cuCtxSetCurrent");
  CUstream s;
  CU_TRY(g_drv.cuStreamCreate(&s, CU_STREAM_NON_BLOCKING), "cuStreamCreate");
  *out = s;
  return EMMY_OK;
}

int emmy_stream_destroy(emmy_stream stream) {
  DRV_OR_FAIL();
  if (stream) CU_TRY(g_drv.cuStreamDestroy(static_cast<CUstream>(stream)), "cuStreamDestroy");
  return EMMY_OK;
}

int emmy_stream_sync(emmy_stream stream) {
  DRV_OR_FAIL();
  CU_TRY(g_drv.cuStreamSynchronize(static_cast<CUstream>(stream)), "cuStreamSynchronize");
  return EMMY_OK;
}

int emmy_event_create(emmy_ctx *ctx, emmy_event *out) {
  if (!ctx || !out) return fail(EMMY_EINVAL, "null argument");
  DRV_OR_FAIL();
  CU_TRY(g_drv.cuCtxSetCurrent(ctx->cu), "cuCtxSetCurrent");
  CUevent e;
  CU_TRY(g_drv.cuEventCreate(&e, CU_EVENT_DEFAULT), "cuEventCreate");
  *out = e;
  return EMMY_OK;
}

int emmy_event_destroy(emmy_event ev) {
  DRV_OR_FAIL();
  if (ev) CU_TRY(g_drv.cuEventDestroy(static_cast<CUevent>(ev)), "cuEventDestroy");
  return EMMY_OK;
}

int emmy_event_record(emmy_event ev, emmy_stream stream) {
  DRV_OR_FAIL();
  CU_TRY(g_drv.cuEventRecord(static_cast<CUevent>(ev), static_cast<CUstream>(stream)), "cuEventRecord");
  return EMMY_OK;
}

int emmy_event_elapsed(emmy_event start, emmy_event end, float *ms) {
  if (!ms) return fail(EMMY_EINVAL, "null ms");
  DRV_OR_FAIL();
  CU_TRY(g_drv.cuEventSynchronize(static_cast<CUevent>(end)), "cuEventSynchronize");
  CU_TRY(g_drv.cuEventElapsedTime(ms, static_cast<CUevent>(start), static_cast<CUevent>(end)),
         "cuEventElapsedTime");
  return EMMY_OK;
}

int emmy_stream_wait_event(emmy_stream stream, emmy_event ev) {
  DRV_OR_FAIL();
  CU_TRY(g_drv.cuStreamWaitEvent(static_cast<CUstream>(stream), static_cast<CUevent>(ev), 0),
         "cuStreamWaitEvent");
  return EMMY_OK;
}

int emmy_error_word(emmy_mod *mod, uint32_t *value, int clear, emmy_stream stream) {
  if (!mod || !value) return fail(EMMY_EINVAL, "null argument");
  emmy_dptr p = 0;
  size_t n = 0;
  int rc = emmy_module_global(mod, "emmy_err", &p, &n);
  if (rc) return rc;
  CU_TRY(g_drv.cuStreamSynchronize(static_cast<CUstream>(stream)), "cuStreamSynchronize");
  uint32_t v = 0;
  CU_TRY(g_drv.cuMemcpyDtoHAsync(&v, p, 4, static_cast<CUstream>(stream)), "cuMemcpyDtoHAsync");
  CU_TRY(g_drv.cuStreamSynchronize(static_cast<CUstream>(stream)), "cuStreamSynchronize");
  *value = v;
  if (clear && v) {
    CU_TRY(g_drv.cuMemsetD32Async(p, 0, 1, static_cast<CUstream>(stream)), "cuMemsetD32Async");
    CU_TRY(g_drv.cuStreamSynchronize(static_cast<CUstream>(stream)), "cuStreamSynchronize");
  }
  return EMMY_OK;
}

int emmy_nccl_unique_id(void *out128) {
  if (!out128) return fail(EMMY_EINVAL, "null argument");
  if (!nccl()) return EMMY_ENONCCL;
  ncclUniqueId id;
  int rc = nc(g_nccl.GetUniqueId(&id), "ncclGetUniqueId");
  if (rc) return rc;
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  memcpy(out128, &id, 128);
  return EMMY_OK;
}

int emmy_nccl_init(emmy_ctx *ctx, int nranks, int rank, const void *id128, emmy_comm **out) {
  if (!ctx || !id128 || !out || nranks < 1 || rank < 0 || rank >= nranks)
    return fail(EMMY_EINVAL, "bad argument");
  DRV_OR_FAIL();
  if (!nccl()) return EMMY_ENONCCL;
  CU_TRY(g_drv.cuCtxSetCurrent(ctx->cu), "cuCtxSetCurrent");
  ncclUniqueId id;
  memcpy(&id, id128, 128);
  auto *c = new emmy_comm();
  int rc = nc(g_nccl.CommInitRank(&c->comm, nranks, id, rank), "ncclCommInitRank");
  if (rc) {
    delete c;
    return rc;
  }
  *out = c;
  return EMMY_OK;
}

int emmy_allreduce_sum_f32(emmy_comm *comm, emmy_dptr buf, size_t count, emmy_stream stream) {
  if (!comm) return fail(EMMY_EINVAL, "null comm");
  if (!nccl()) return EMMY_ENONCCL;
  void *p = reinterpret_cast<void *>(buf);
  return nc(g_nccl.AllReduce(p, p, count, ncclFloat32, ncclSum, comm->comm,
                             static_cast<cudaStream_t>(stream)),
            "ncclAllReduce");
}

int emmy_nccl_async_error(emmy_comm *comm, int *nccl_result) {
  if (!comm || !nccl_result) return fail(EMMY_EINVAL, "null argument");
  if (!nccl()) return EMMY_ENONCCL;
  ncclResult_t r = ncclSuccess;
  int rc = nc(g_nccl.CommGetAsyncError(comm->comm, &r), "ncclCommGetAsyncError");
  *nccl_result = int(r);
  return rc;
}

int emmy_nccl_abort(emmy_comm *comm) {
  if (!comm) return EMMY_OK;
  if (!nccl()) return EMMY_ENONCCL;
  int rc = nc(g_nccl.CommAbort(comm->comm), "ncclCommAbort");
  delete comm;
  return rc;
}

int emmy_nccl_destroy(emmy_comm *comm) {
  if (!comm) return EMMY_OK;
  if (!nccl()) return EMMY_ENONCCL;
  int rc = nc(g_nccl.CommDestroy(comm->comm), "ncclCommDestroy");
  delete comm;
  return rc;
}

}  // extern "C"
