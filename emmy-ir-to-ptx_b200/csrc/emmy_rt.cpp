// emmy_rt.cpp -- B200 runtime for the PTX emitted by compile.py (C ABI in
// include/emmy_rt.h).
//
// The driver API is resolved with dlopen/dlsym at first use, so this library
// links and loads without a GPU or driver; the entry points then report
// EMMY_RT_ENODRIVER. Only documented driver entry points are used, one
// cudaMemcpy-equivalent per buffer (no batched copy calls).

#include "emmy_rt.h"

#include <cuda.h>
#include <dlfcn.h>

#include <algorithm>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace {

thread_local char g_err[2048] = "";

int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

struct Driver {
  bool ok = false;
  std::string why;
#define EMMY_FN(name, ret, args) ret(CUDAAPI *name) args = nullptr;
  EMMY_FN(Init, CUresult, (unsigned int))
  EMMY_FN(DeviceGet, CUresult, (CUdevice *, int))
  EMMY_FN(DeviceGetAttribute, CUresult, (int *, CUdevice_attribute, CUdevice))
  EMMY_FN(DeviceGetName, CUresult, (char *, int, CUdevice))
  EMMY_FN(DevicePrimaryCtxRetain, CUresult, (CUcontext *, CUdevice))
  EMMY_FN(CtxSetCurrent, CUresult, (CUcontext))
  EMMY_FN(CtxGetCurrent, CUresult, (CUcontext *))
  EMMY_FN(ModuleLoadDataEx, CUresult, (CUmodule *, const void *, unsigned int, CUjit_option *, void **))
  EMMY_FN(ModuleUnload, CUresult, (CUmodule))
  EMMY_FN(ModuleGetFunction, CUresult, (CUfunction *, CUmodule, const char *))
  EMMY_FN(ModuleGetGlobal, CUresult, (CUdeviceptr *, size_t *, CUmodule, const char *))
  EMMY_FN(FuncGetAttribute, CUresult, (int *, CUfunction_attribute, CUfunction))
  EMMY_FN(FuncSetAttribute, CUresult, (CUfunction, CUfunction_attribute, int))
  EMMY_FN(LaunchKernel, CUresult, (CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, CUstream, void **, void **))
  EMMY_FN(LaunchKernelEx, CUresult, (const CUlaunchConfig *, CUfunction, void **, void **))
  EMMY_FN(MemAlloc, CUresult, (CUdeviceptr *, size_t))
  EMMY_FN(MemFree, CUresult, (CUdeviceptr))
  EMMY_FN(MemcpyHtoD, CUresult, (CUdeviceptr, const void *, size_t))
  EMMY_FN(MemcpyDtoH, CUresult, (void *, CUdeviceptr, size_t))
  EMMY_FN(MemcpyHtoDAsync, CUresult, (CUdeviceptr, const void *, size_t, CUstream))
  EMMY_FN(MemcpyDtoHAsync, CUresult, (void *, CUdeviceptr, size_t, CUstream))
  EMMY_FN(MemsetD8, CUresult, (CUdeviceptr, unsigned char, size_t))
  EMMY_FN(MemsetD8Async, CUresult, (CUdeviceptr, unsigned char, size_t, CUstream))
  EMMY_FN(MemsetD32Async, CUresult, (CUdeviceptr, unsigned int, size_t, CUstream))
  EMMY_FN(MemHostAlloc, CUresult, (void **, size_t, unsigned int))
  EMMY_FN(MemFreeHost, CUresult, (void *))
  EMMY_FN(EventCreate, CUresult, (CUevent *, unsigned int))
  EMMY_FN(EventRecord, CUresult, (CUevent, CUstream))
  EMMY_FN(EventSynchronize, CUresult, (CUevent))
  EMMY_FN(EventQuery, CUresult, (CUevent))
  EMMY_FN(EventElapsedTime, CUresult, (float *, CUevent, CUevent))
  EMMY_FN(EventDestroy, CUresult, (CUevent))
  EMMY_FN(StreamCreate, CUresult, (CUstream *, unsigned int))
  EMMY_FN(StreamDestroy, CUresult, (CUstream))
  EMMY_FN(StreamQuery, CUresult, (CUstream))
  EMMY_FN(GetErrorString, CUresult, (CUresult, const char **))
  // optional: without them modules keep their register-staged loads
  EMMY_FN(TensorMapEncodeTiled, CUresult,
          (CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
           const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
           CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill))
  EMMY_FN(StreamIsCapturing, CUresult, (CUstream, CUstreamCaptureStatus *))
  EMMY_FN(CtxSynchronize, CUresult, (void))
#undef EMMY_FN
};

Driver g_drv;
std::once_flag g_once;

template <class T>
bool bind(void *h, T &fn, const char *sym, std::string &missing) {
  fn = reinterpret_cast<T>(dlsym(h, sym));
  if (!fn) missing += std::string(" ") + sym;
  return fn != nullptr;
}

void load_driver() {
  void *h = dlopen("libcuda.so.1", RTLD_NOW | RTLD_LOCAL);
  if (!h) h = dlopen("libcuda.so", RTLD_NOW | RTLD_LOCAL);
  if (!h) {
    g_drv.why = std::string("cannot load libcuda.so.1: ") + dlerror();
    return;
  }
  std::string m;
  Driver &d = g_drv;
  bind(h, d.Init, "cuInit", m);
  bind(h, d.DeviceGet, "cuDeviceGet", m);
  bind(h, d.DeviceGetAttribute, "cuDeviceGetAttribute", m);
  bind(h, d.DeviceGetName, "cuDeviceGetName", m);
  bind(h, d.DevicePrimaryCtxRetain, "cuDevicePrimaryCtxRetain", m);
  bind(h, d.CtxSetCurrent, "cuCtxSetCurrent", m);
  bind(h, d.CtxGetCurrent, "cuCtxGetCurrent", m);
  bind(h, d.ModuleLoadDataEx, "cuModuleLoadDataEx", m);
  bind(h, d.ModuleUnload, "cuModuleUnload", m);
  bind(h, d.ModuleGetFunction, "cuModuleGetFunction", m);
  bind(h, d.ModuleGetGlobal, "cuModuleGetGlobal_v2", m);
  bind(h, d.FuncGetAttribute, "cuFuncGetAttribute", m);
  bind(h, d.FuncSetAttribute, "cuFuncSetAttribute", m);
  bind(h, d.LaunchKernel, "cuLaunchKernel", m);
  bind(h, d.LaunchKernelEx, "cuLaunchKernelEx", m);
  bind(h, d.MemAlloc, "cuMemAlloc_v2", m);
  bind(h, d.MemFree, "cuMemFree_v2", m);
  bind(h, d.MemcpyHtoD, "cuMemcpyHtoD_v2", m);
  bind(h, d.MemcpyDtoH, "cuMemcpyDtoH_v2", m);
  bind(h, d.MemcpyHtoDAsync, "cuMemcpyHtoDAsync_v2", m);
  bind(h, d.MemcpyDtoHAsync, "cuMemcpyDtoHAsync_v2", m);
  bind(h, d.MemsetD8, "cuMemsetD8_v2", m);
  bind(h, d.MemsetD8Async, "cuMemsetD8Async", m);
  bind(h, d.MemsetD32Async, "cuMemsetD32Async", m);
  bind(h, d.MemHostAlloc, "cuMemHostAlloc", m);
  bind(h, d.MemFreeHost, "cuMemFreeHost", m);
  bind(h, d.EventCreate, "cuEventCreate", m);
  bind(h, d.EventRecord, "cuEventRecord", m);
  bind(h, d.EventSynchronize, "cuEventSynchronize", m);
  bind(h, d.EventQuery, "cuEventQuery", m);
  bind(h, d.EventElapsedTime, "cuEventElapsedTime", m);
  bind(h, d.EventDestroy, "cuEventDestroy_v2", m);
  bind(h, d.StreamCreate, "cuStreamCreate", m);
  bind(h, d.StreamDestroy, "cuStreamDestroy_v2", m);
  bind(h, d.StreamQuery, "cuStreamQuery", m);
  bind(h, d.GetErrorString, "cuGetErrorString", m);
  std::string optional;
  bind(h, d.TensorMapEncodeTiled, "cuTensorMapEncodeTiled", optional);
  bind(h, d.StreamIsCapturing, "cuStreamIsCapturing", optional);
  bind(h, d.CtxSynchronize, "cuCtxSynchronize", optional);
  if (!m.empty()) {
    g_drv.why = "libcuda.so.1 lacks:" + m;
    return;
  }
  g_drv.ok = true;
}

int need_driver() {
  std::call_once(g_once, load_driver);
  if (!g_drv.ok) return fail(EMMY_RT_ENODRIVER, "%s", g_drv.why.c_str());
  return EMMY_RT_OK;
}

int cu_check(CUresult r, const char *what) {
  if (r == CUDA_SUCCESS) return EMMY_RT_OK;
  const char *s = nullptr;
  if (g_drv.GetErrorString) g_drv.GetErrorString(r, &s);
  return fail(EMMY_RT_ECUDA, "%s failed: %s (%d)", what, s ? s : "unknown error", int(r));
}

#define CU(call, what)                              \
  do {                                              \
    int _rc = cu_check((call), (what));             \
    if (_rc) return _rc;                            \
  } while (0)

thread_local int g_device = -1;

int ensure_context() {
  int rc = need_driver();
  if (rc) return rc;
  CUcontext cur = nullptr;
  CU(g_drv.CtxGetCurrent(&cur), "cuCtxGetCurrent");
  if (cur) return EMMY_RT_OK;
  return emmy_rt_init(g_device < 0 ? 0 : g_device);
}

}  // namespace

// Lets other translation units of this library report through emmy_rt_last_error().
__attribute__((visibility("hidden"))) void emmy_rt_internal_set_error(const char *msg) {
  snprintf(g_err, sizeof(g_err), "%s", msg ? msg : "");
}

// Tensor maps a module asks the runtime to write before its launches. The compiler declares
// emmy_tmap_desc (what to encode), emmy_tmap (the maps) and emmy_tmap_key (the pointer each
// map was encoded for); the kernel compares the keys with its own parameters and takes its
// TMA path only when they all match, so a stale or missing map costs speed, never results.
// A map is rewritten only when a launch's pointers differ from the keys, and only after every
// earlier launch of the module has finished (so no running kernel reads a map being written);
// the copies go on the launch stream in front of the kernel, maps before keys.
constexpr uint32_t kTmapMagic = 0x454D5401u;
constexpr int kTmapWords = 24;
constexpr int kTmapMax = 4;

struct TensorMaps {
  int n = 0;                      // maps the module declares (0: none)
  uint32_t desc[kTmapWords * kTmapMax] = {};
  CUdeviceptr maps = 0, keys = 0;
  uint64_t key[kTmapMax] = {};    // host copy of the device keys
  int enabled = 1;
  int frozen = 0;                 // launched under stream capture: never rewritten again
  uint64_t uploads = 0;
  std::vector<std::pair<CUstream, CUevent>> launched;   // last launch per stream
  alignas(64) CUtensorMap staged[kTmapMax];
  uint64_t staged_keys[kTmapMax] = {};
  std::mutex lock;                // launches of one module from several host threads
};

struct emmy_module {
  CUmodule mod = nullptr;
  CUfunction fn = nullptr;
  int dyn_smem_set = 0;
  TensorMaps tm;
};

namespace {

// Reads the module's tensor-map table, if it has one. A table that is present but malformed
// is an error (only this compiler writes it).
int tmap_setup(emmy_module *m) {
  CUdeviceptr p = 0;
  size_t n = 0;
  CUresult r = g_drv.ModuleGetGlobal(&p, &n, m->mod, "emmy_tmap_desc");
  if (r == CUDA_ERROR_NOT_FOUND) return EMMY_RT_OK;
  CU(r, "cuModuleGetGlobal(emmy_tmap_desc)");
  uint32_t head[2] = {0, 0};
  if (n < sizeof(head)) return fail(EMMY_RT_EINVAL, "tensor-map table too short");
  CU(g_drv.MemcpyDtoH(head, p, sizeof(head)), "cuMemcpyDtoH");
  int count = int(head[1]);
  if (head[0] != kTmapMagic || count < 1 || count > kTmapMax ||
      n < sizeof(head) + size_t(count) * kTmapWords * 4)
    return fail(EMMY_RT_EINVAL, "malformed tensor-map table");
  TensorMaps &t = m->tm;
  CU(g_drv.MemcpyDtoH(t.desc, p + sizeof(head), size_t(count) * kTmapWords * 4),
     "cuMemcpyDtoH");
  size_t bm = 0, bk = 0;
  CU(g_drv.ModuleGetGlobal(&t.maps, &bm, m->mod, "emmy_tmap"), "cuModuleGetGlobal(emmy_tmap)");
  CU(g_drv.ModuleGetGlobal(&t.keys, &bk, m->mod, "emmy_tmap_key"),
     "cuModuleGetGlobal(emmy_tmap_key)");
  if (bm < size_t(count) * 128 || bk < size_t(count) * 8 || (t.maps & 63))
    return fail(EMMY_RT_EINVAL, "tensor-map globals too small or misaligned");
  for (int k = 0; k < count; ++k) {
    uint32_t rank = t.desc[k * kTmapWords + 1];
    if (rank < 1 || rank > 5) return fail(EMMY_RT_EINVAL, "tensor-map rank out of range");
  }
  t.n = g_drv.TensorMapEncodeTiled && g_drv.StreamIsCapturing && g_drv.CtxSynchronize ? count : 0;
  return EMMY_RT_OK;
}

bool tmap_encode(const uint32_t *d, uint64_t ptr, CUtensorMap *out) {
  cuuint32_t rank = d[1];
  cuuint64_t dims[5], strides[4];
  cuuint32_t box[5], estr[5];
  for (int i = 0; i < 5; ++i) {
    dims[i] = d[2 + i];
    box[i] = d[15 + i];
    estr[i] = 1;
  }
  for (int i = 0; i < 4; ++i)
    strides[i] = cuuint64_t(d[7 + 2 * i]) | (cuuint64_t(d[8 + 2 * i]) << 32);
  return g_drv.TensorMapEncodeTiled(out, CUtensorMapDataType(d[21]), rank,
                                    reinterpret_cast<void *>(static_cast<uintptr_t>(ptr)), dims,
                                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                    CUtensorMapSwizzle(d[20]), CUtensorMapL2promotion(d[22]),
                                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Before a launch: bring the device maps in line with this launch's pointers when that is
// safe. Sets *track when the launch is to be recorded for later updates.
int tmap_prepare(emmy_module *m, const uint64_t *args, int nargs, CUstream s, bool *track) {
  TensorMaps &t = m->tm;
  *track = false;
  if (!t.n || !t.enabled) return EMMY_RT_OK;
  CUstreamCaptureStatus cap = CU_STREAM_CAPTURE_STATUS_NONE;
  CU(g_drv.StreamIsCapturing(s, &cap), "cuStreamIsCapturing");
  if (cap != CU_STREAM_CAPTURE_STATUS_NONE) {
    t.frozen = 1;   // a graph may replay this launch at any time from now on
    return EMMY_RT_OK;
  }
  *track = true;
  uint64_t want[kTmapMax] = {};
  bool same = true;
  for (int k = 0; k < t.n; ++k) {
    uint32_t idx = t.desc[k * kTmapWords];
    if (int(idx) >= nargs) return EMMY_RT_OK;
    want[k] = args[idx];
    same = same && want[k] == t.key[k];
  }
  if (same || t.frozen) return EMMY_RT_OK;
  for (int k = 0; k < t.n; ++k)
    if (!tmap_encode(&t.desc[k * kTmapWords], want[k], &t.staged[k]))
      return EMMY_RT_OK;   // e.g. a pointer that is not 16-byte aligned: no TMA for it
  for (auto &e : t.launched) CU(g_drv.EventSynchronize(e.second), "cuEventSynchronize");
  std::memcpy(t.staged_keys, want, sizeof(want));
  CU(g_drv.MemcpyHtoDAsync(t.maps, t.staged, size_t(t.n) * 128, s), "cuMemcpyHtoDAsync");
  CU(g_drv.MemcpyHtoDAsync(t.keys, t.staged_keys, size_t(t.n) * 8, s), "cuMemcpyHtoDAsync");
  std::memcpy(t.key, want, sizeof(want));
  ++t.uploads;
  return EMMY_RT_OK;
}

// After a launch: remember it, per stream, so a later rewrite can wait for it. Entries whose
// launch has finished are dropped first (a host that makes a stream per call, as emmy_rt_run
// does, would otherwise grow the list without bound).
int tmap_track(emmy_module *m, CUstream s) {
  TensorMaps &t = m->tm;
  for (auto &e : t.launched)
    if (e.first == s) return cu_check(g_drv.EventRecord(e.second, s), "cuEventRecord");
  for (size_t i = 0; i < t.launched.size();) {
    if (g_drv.EventQuery(t.launched[i].second) == CUDA_SUCCESS) {
      g_drv.EventDestroy(t.launched[i].second);
      t.launched[i] = t.launched.back();
      t.launched.pop_back();
    } else {
      ++i;
    }
  }
  CUevent ev = nullptr;
  CU(g_drv.EventCreate(&ev, CU_EVENT_DISABLE_TIMING), "cuEventCreate");
  t.launched.emplace_back(s, ev);
  return cu_check(g_drv.EventRecord(ev, s), "cuEventRecord");
}

void tmap_release(emmy_module *m) {
  for (auto &e : m->tm.launched) g_drv.EventDestroy(e.second);
  m->tm.launched.clear();
}

}  // namespace

extern "C" {

int emmy_rt_abi_version(void) { return EMMY_RT_ABI_VERSION; }

const char *emmy_rt_last_error(void) { return g_err; }

int emmy_rt_init(int device) {
  int rc = need_driver();
  if (rc) return rc;
  CU(g_drv.Init(0), "cuInit");
  CUdevice dev;
  CU(g_drv.DeviceGet(&dev, device), "cuDeviceGet");
  CUcontext ctx;
  CU(g_drv.DevicePrimaryCtxRetain(&ctx, dev), "cuDevicePrimaryCtxRetain");
  CU(g_drv.CtxSetCurrent(ctx), "cuCtxSetCurrent");
  g_device = device;
  return EMMY_RT_OK;
}

int emmy_rt_device_info(int device, int *sm_count, int *cc_major, int *cc_minor, int *l2_bytes,
                        int *max_smem_optin, char *name, size_t name_size) {
  int rc = need_driver();
  if (rc) return rc;
  CU(g_drv.Init(0), "cuInit");
  CUdevice dev;
  CU(g_drv.DeviceGet(&dev, device), "cuDeviceGet");
  int v;
  if (sm_count) {
    CU(g_drv.DeviceGetAttribute(&v, CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT, dev), "attr");
    *sm_count = v;
  }
  if (cc_major) {
    CU(g_drv.DeviceGetAttribute(&v, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MAJOR, dev), "attr");
    *cc_major = v;
  }
  if (cc_minor) {
    CU(g_drv.DeviceGetAttribute(&v, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MINOR, dev), "attr");
    *cc_minor = v;
  }
  if (l2_bytes) {
    CU(g_drv.DeviceGetAttribute(&v, CU_DEVICE_ATTRIBUTE_L2_CACHE_SIZE, dev), "attr");
    *l2_bytes = v;
  }
  if (max_smem_optin) {
    CU(g_drv.DeviceGetAttribute(&v, CU_DEVICE_ATTRIBUTE_MAX_SHARED_MEMORY_PER_BLOCK_OPTIN, dev),
       "attr");
    *max_smem_optin = v;
  }
  if (name && name_size) CU(g_drv.DeviceGetName(name, int(name_size), dev), "cuDeviceGetName");
  return EMMY_RT_OK;
}

int emmy_rt_module_load(const char *ptx, const char *entry, emmy_module **out, char *log,
                        size_t log_size) {
  if (!ptx || !entry || !out) return fail(EMMY_RT_EINVAL, "null argument");
  int rc = ensure_context();
  if (rc) return rc;
  std::vector<char> errlog(16384, 0);
  CUjit_option opts[2] = {CU_JIT_ERROR_LOG_BUFFER, CU_JIT_ERROR_LOG_BUFFER_SIZE_BYTES};
  void *vals[2] = {errlog.data(), reinterpret_cast<void *>(static_cast<uintptr_t>(errlog.size()))};
  CUmodule mod = nullptr;
  CUresult r = g_drv.ModuleLoadDataEx(&mod, ptx, 2, opts, vals);
  if (log && log_size) {
    std::strncpy(log, errlog.data(), log_size - 1);
    log[log_size - 1] = '\0';
  }
  if (r != CUDA_SUCCESS) {
    cu_check(r, "cuModuleLoadDataEx");
    return fail(EMMY_RT_ECUDA, "PTX JIT failed (%d): %s", int(r), errlog.data());
  }
  CUfunction fn = nullptr;
  r = g_drv.ModuleGetFunction(&fn, mod, entry);
  if (r != CUDA_SUCCESS) {
    g_drv.ModuleUnload(mod);
    return fail(EMMY_RT_ENOTFOUND, "entry %s not found in module", entry);
  }
  emmy_module *m = new emmy_module;
  m->mod = mod;
  m->fn = fn;
  rc = tmap_setup(m);
  if (rc) {
    g_drv.ModuleUnload(mod);
    delete m;
    return rc;
  }
  *out = m;
  return EMMY_RT_OK;
}

int emmy_rt_module_unload(emmy_module *m) {
  if (!m) return EMMY_RT_OK;
  int rc = need_driver();
  if (rc) return rc;
  tmap_release(m);
  CUresult r = g_drv.ModuleUnload(m->mod);
  delete m;
  return cu_check(r, "cuModuleUnload");
}

int emmy_rt_module_attrs(emmy_module *m, int *num_regs, int *static_smem, int *max_threads) {
  if (!m) return fail(EMMY_RT_EINVAL, "null module");
  int rc = need_driver();
  if (rc) return rc;
  if (num_regs) CU(g_drv.FuncGetAttribute(num_regs, CU_FUNC_ATTRIBUTE_NUM_REGS, m->fn), "attr");
  if (static_smem)
    CU(g_drv.FuncGetAttribute(static_smem, CU_FUNC_ATTRIBUTE_SHARED_SIZE_BYTES, m->fn), "attr");
  if (max_threads)
    CU(g_drv.FuncGetAttribute(max_threads, CU_FUNC_ATTRIBUTE_MAX_THREADS_PER_BLOCK, m->fn),
       "attr");
  return EMMY_RT_OK;
}

int emmy_rt_module_global(emmy_module *m, const char *name, uint64_t *dptr, uint64_t *bytes) {
  if (!m || !name) return fail(EMMY_RT_EINVAL, "null argument");
  int rc = need_driver();
  if (rc) return rc;
  CUdeviceptr p = 0;
  size_t n = 0;
  CUresult r = g_drv.ModuleGetGlobal(&p, &n, m->mod, name);
  if (r == CUDA_ERROR_NOT_FOUND) return fail(EMMY_RT_ENOTFOUND, "no global %s", name);
  CU(r, "cuModuleGetGlobal");
  if (dptr) *dptr = p;
  if (bytes) *bytes = n;
  return EMMY_RT_OK;
}

int emmy_rt_module_error_word(emmy_module *m, uint32_t *value, int clear) {
  uint64_t p = 0, n = 0;
  int rc = emmy_rt_module_global(m, "emmy_error", &p, &n);
  if (rc == EMMY_RT_ENOTFOUND) {
    if (value) *value = 0;
    g_err[0] = '\0';
    return EMMY_RT_OK;
  }
  if (rc) return rc;
  uint32_t v = 0;
  CU(g_drv.MemcpyDtoH(&v, p, sizeof(v)), "cuMemcpyDtoH");
  if (value) *value = v;
  if (clear && v) CU(g_drv.MemsetD8(p, 0, sizeof(v)), "cuMemsetD8");
  return EMMY_RT_OK;
}

int emmy_rt_module_tensor_maps(emmy_module *m, int enable, int *nmaps, uint64_t *uploads) {
  if (!m) return fail(EMMY_RT_EINVAL, "null module");
  if (enable < -1 || enable > 1) return fail(EMMY_RT_EINVAL, "enable must be -1, 0 or 1");
  int rc = ensure_context();
  if (rc) return rc;
  TensorMaps &t = m->tm;
  std::lock_guard<std::mutex> guard(t.lock);
  if (enable == 0 && t.n && t.enabled) {
    for (auto &e : t.launched) CU(g_drv.EventSynchronize(e.second), "cuEventSynchronize");
    CU(g_drv.MemsetD8(t.keys, 0, size_t(t.n) * 8), "cuMemsetD8");
    CU(g_drv.CtxSynchronize(), "cuCtxSynchronize");
    std::memset(t.key, 0, sizeof(t.key));
    t.enabled = 0;
  } else if (enable == 1) {
    t.enabled = 1;
  }
  if (nmaps) *nmaps = t.n;
  if (uploads) *uploads = t.uploads;
  return EMMY_RT_OK;
}

static int launch_raw(emmy_module *m, const uint32_t grid[3], const uint32_t block[3],
                      uint32_t smem_bytes, const uint64_t *args, int nargs, CUstream stream,
                      uint32_t flags = 0) {
  if (smem_bytes > 48 * 1024 && int(smem_bytes) != m->dyn_smem_set) {
    CU(g_drv.FuncSetAttribute(m->fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                              int(smem_bytes)),
       "cuFuncSetAttribute(MAX_DYNAMIC_SHARED_SIZE_BYTES)");
    m->dyn_smem_set = int(smem_bytes);
  }
  bool track = false;
  // a module with tensor maps: its keys, maps and launch records change together with the
  // launch that needs them
  std::unique_lock<std::mutex> guard;
  if (m->tm.n) guard = std::unique_lock<std::mutex>(m->tm.lock);
  int trc = tmap_prepare(m, args, nargs, stream, &track);
  if (trc) return trc;
  std::vector<uint64_t> vals(args, args + nargs);
  std::vector<void *> params(static_cast<size_t>(nargs));
  for (int i = 0; i < nargs; ++i) params[size_t(i)] = &vals[size_t(i)];
  if (flags & EMMY_RT_LAUNCH_OVERLAP) {
    // programmatic stream serialization: this grid may start once every CTA of the
    // previous kernel on the stream has run griddepcontrol.launch_dependents; it orders
    // itself after that kernel with griddepcontrol.wait where it needs to
    CUlaunchAttribute attr;
    std::memset(&attr, 0, sizeof(attr));
    attr.id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
    attr.value.programmaticStreamSerializationAllowed = 1;
    CUlaunchConfig cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDimX = grid[0];
    cfg.gridDimY = grid[1];
    cfg.gridDimZ = grid[2];
    cfg.blockDimX = block[0];
    cfg.blockDimY = block[1];
    cfg.blockDimZ = block[2];
    cfg.sharedMemBytes = smem_bytes;
    cfg.hStream = stream;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    CU(g_drv.LaunchKernelEx(&cfg, m->fn, nargs ? params.data() : nullptr, nullptr),
       "cuLaunchKernelEx");
  } else {
    CU(g_drv.LaunchKernel(m->fn, grid[0], grid[1], grid[2], block[0], block[1], block[2],
                          smem_bytes, stream, nargs ? params.data() : nullptr, nullptr),
       "cuLaunchKernel");
  }
  return track ? tmap_track(m, stream) : EMMY_RT_OK;
}

int emmy_rt_launch(emmy_module *m, const uint32_t grid[3], const uint32_t block[3],
                   uint32_t smem_bytes, const uint64_t *args, int nargs, uint64_t stream) {
  if (!m || !grid || !block || (nargs && !args)) return fail(EMMY_RT_EINVAL, "null argument");
  int rc = ensure_context();
  if (rc) return rc;
  return launch_raw(m, grid, block, smem_bytes, args, nargs,
                    reinterpret_cast<CUstream>(static_cast<uintptr_t>(stream)));
}

int emmy_rt_launch_ex(emmy_module *m, const uint32_t grid[3], const uint32_t block[3],
                      uint32_t smem_bytes, const uint64_t *args, int nargs, uint64_t stream,
                      uint32_t flags) {
  if (!m || !grid || !block || (nargs && !args)) return fail(EMMY_RT_EINVAL, "null argument");
  if (flags & ~uint32_t(EMMY_RT_LAUNCH_OVERLAP)) return fail(EMMY_RT_EINVAL, "unknown flags");
  int rc = ensure_context();
  if (rc) return rc;
  return launch_raw(m, grid, block, smem_bytes, args, nargs,
                    reinterpret_cast<CUstream>(static_cast<uintptr_t>(stream)), flags);
}

int emmy_rt_sync(uint64_t stream, int timeout_ms) {
  int rc = ensure_context();
  if (rc) return rc;
  CUstream s = reinterpret_cast<CUstream>(static_cast<uintptr_t>(stream));
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    CUresult r = g_drv.StreamQuery(s);
    if (r == CUDA_SUCCESS) return EMMY_RT_OK;
    if (r != CUDA_ERROR_NOT_READY) return cu_check(r, "cuStreamQuery");
    auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                  std::chrono::steady_clock::now() - t0)
                  .count();
    if (timeout_ms >= 0 && ms > timeout_ms)
      return fail(EMMY_RT_ETIMEOUT, "stream did not finish within %d ms", timeout_ms);
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

namespace {
struct Events {
  std::vector<CUevent> ev;
  ~Events() {
    for (CUevent e : ev)
      if (e) g_drv.EventDestroy(e);
  }
  int make(size_t n) {
    ev.assign(n, nullptr);
    for (auto &e : ev) CU(g_drv.EventCreate(&e, CU_EVENT_DEFAULT), "cuEventCreate");
    return EMMY_RT_OK;
  }
};
}  // namespace

int emmy_rt_time(emmy_module *m, const uint32_t grid[3], const uint32_t block[3],
                 uint32_t smem_bytes, const uint64_t *args, int nargs, uint64_t stream,
                 int warmup, int iters, uint64_t flush_ptr, uint64_t flush_bytes,
                 float *ms_out) {
  if (!m || iters <= 0 || !ms_out) return fail(EMMY_RT_EINVAL, "bad argument");
  int rc = ensure_context();
  if (rc) return rc;
  CUstream s = reinterpret_cast<CUstream>(static_cast<uintptr_t>(stream));
  for (int i = 0; i < warmup; ++i) {
    if (flush_bytes) CU(g_drv.MemsetD32Async(flush_ptr, 0x3f800000u + i, flush_bytes / 4, s), "flush");
    rc = launch_raw(m, grid, block, smem_bytes, args, nargs, s);
    if (rc) return rc;
  }
  Events e;
  rc = e.make(size_t(2 * iters));
  if (rc) return rc;
  for (int i = 0; i < iters; ++i) {
    if (flush_bytes) CU(g_drv.MemsetD32Async(flush_ptr, 0x40000000u + i, flush_bytes / 4, s), "flush");
    CU(g_drv.EventRecord(e.ev[size_t(2 * i)], s), "cuEventRecord");
    rc = launch_raw(m, grid, block, smem_bytes, args, nargs, s);
    if (rc) return rc;
    CU(g_drv.EventRecord(e.ev[size_t(2 * i + 1)], s), "cuEventRecord");
  }
  rc = emmy_rt_sync(stream, 120000);
  if (rc) return rc;
  for (int i = 0; i < iters; ++i)
    CU(g_drv.EventElapsedTime(&ms_out[i], e.ev[size_t(2 * i)], e.ev[size_t(2 * i + 1)]),
       "cuEventElapsedTime");
  return EMMY_RT_OK;
}

static float median(std::vector<float> v) {
  if (v.empty()) return 0.f;
  std::sort(v.begin(), v.end());
  size_t n = v.size();
  return n % 2 ? v[n / 2] : 0.5f * (v[n / 2 - 1] + v[n / 2]);
}

int emmy_rt_run(emmy_module *m, const uint32_t grid[3], const uint32_t block[3],
                uint32_t smem_bytes, emmy_arg *args, int nargs, int warmup, int iters,
                emmy_run_stats *stats) {
  if (!m || !grid || !block || nargs < 0 || (nargs && !args) || iters <= 0)
    return fail(EMMY_RT_EINVAL, "bad argument");
  int rc = ensure_context();
  if (rc) return rc;
  std::vector<CUdeviceptr> dev(static_cast<size_t>(nargs), 0);
  struct Guard {
    std::vector<CUdeviceptr> *d;
    CUstream s = nullptr;
    ~Guard() {
      for (CUdeviceptr p : *d)
        if (p) g_drv.MemFree(p);
      if (s) g_drv.StreamDestroy(s);
    }
  } guard{&dev};
  std::vector<uint64_t> ptrs(static_cast<size_t>(nargs));
  uint64_t h2d = 0, d2h = 0;
  for (int i = 0; i < nargs; ++i) {
    size_t n = std::max<uint64_t>(args[i].bytes, 4);
    CU(g_drv.MemAlloc(&dev[size_t(i)], n), "cuMemAlloc");
    CU(g_drv.MemsetD8(dev[size_t(i)], 0, n), "cuMemsetD8");
    ptrs[size_t(i)] = dev[size_t(i)];
    if (args[i].is_output)
      d2h += args[i].bytes;
    else
      h2d += args[i].bytes;
  }
  CU(g_drv.StreamCreate(&guard.s, CU_STREAM_NON_BLOCKING), "cuStreamCreate");
  CUstream s = guard.s;
  Events e;
  rc = e.make(4);
  if (rc) return rc;
  std::vector<float> ker, e2e;
  for (int it = 0; it < warmup + iters; ++it) {
    CU(g_drv.EventRecord(e.ev[0], s), "cuEventRecord");
    for (int i = 0; i < nargs; ++i) {
      if (args[i].is_output) {
        if (args[i].zero_each && it > 0)
          CU(g_drv.MemsetD8Async(dev[size_t(i)], 0, args[i].bytes, s), "cuMemsetD8Async");
      } else if (args[i].bytes) {
        CU(g_drv.MemcpyHtoDAsync(dev[size_t(i)], args[i].host, args[i].bytes, s),
           "cuMemcpyHtoDAsync");
      }
    }
    CU(g_drv.EventRecord(e.ev[1], s), "cuEventRecord");
    rc = launch_raw(m, grid, block, smem_bytes, ptrs.data(), nargs, s);
    if (rc) return rc;
    CU(g_drv.EventRecord(e.ev[2], s), "cuEventRecord");
    for (int i = 0; i < nargs; ++i)
      if (args[i].is_output && args[i].bytes)
        CU(g_drv.MemcpyDtoHAsync(args[i].host, dev[size_t(i)], args[i].bytes, s),
           "cuMemcpyDtoHAsync");
    CU(g_drv.EventRecord(e.ev[3], s), "cuEventRecord");
    rc = emmy_rt_sync(static_cast<uint64_t>(reinterpret_cast<uintptr_t>(s)), 120000);
    if (rc) return rc;
    if (it >= warmup) {
      float a = 0, b = 0;
      CU(g_drv.EventElapsedTime(&a, e.ev[1], e.ev[2]), "cuEventElapsedTime");
      CU(g_drv.EventElapsedTime(&b, e.ev[0], e.ev[3]), "cuEventElapsedTime");
      ker.push_back(a * 1000.f);
      e2e.push_back(b * 1000.f);
    }
  }
  if (stats) {
    stats->kernel_us_median = median(ker);
    stats->e2e_us_median = median(e2e);
    stats->h2d_bytes = h2d;
    stats->d2h_bytes = d2h;
    stats->iters = iters;
  }
  return EMMY_RT_OK;
}

int emmy_rt_mem_alloc(uint64_t bytes, uint64_t *dptr) {
  if (!dptr) return fail(EMMY_RT_EINVAL, "null argument");
  int rc = ensure_context();
  if (rc) return rc;
  CUdeviceptr p = 0;
  CU(g_drv.MemAlloc(&p, size_t(std::max<uint64_t>(bytes, 4))), "cuMemAlloc");
  *dptr = p;
  return EMMY_RT_OK;
}

int emmy_rt_mem_free(uint64_t dptr) {
  int rc = ensure_context();
  if (rc) return rc;
  return cu_check(g_drv.MemFree(dptr), "cuMemFree");
}

int emmy_rt_memcpy_htod(uint64_t dst, const void *src, uint64_t bytes) {
  int rc = ensure_context();
  if (rc) return rc;
  return cu_check(g_drv.MemcpyHtoD(dst, src, size_t(bytes)), "cuMemcpyHtoD");
}

int emmy_rt_memcpy_dtoh(void *dst, uint64_t src, uint64_t bytes) {
  int rc = ensure_context();
  if (rc) return rc;
  return cu_check(g_drv.MemcpyDtoH(dst, src, size_t(bytes)), "cuMemcpyDtoH");
}

int emmy_rt_memset_zero(uint64_t dptr, uint64_t bytes) {
  int rc = ensure_context();
  if (rc) return rc;
  return cu_check(g_drv.MemsetD8(dptr, 0, size_t(bytes)), "cuMemsetD8");
}

int emmy_rt_host_alloc(uint64_t bytes, void **ptr) {
  if (!ptr) return fail(EMMY_RT_EINVAL, "null argument");
  int rc = ensure_context();
  if (rc) return rc;
  return cu_check(g_drv.MemHostAlloc(ptr, size_t(std::max<uint64_t>(bytes, 4)), 0),
                  "cuMemHostAlloc");
}

int emmy_rt_host_free(void *ptr) {
  int rc = ensure_context();
  if (rc) return rc;
  return cu_check(g_drv.MemFreeHost(ptr), "cuMemFreeHost");
}

}  // extern "C"
