// libtgcb runtime: NVRTC compilation, module loading and plan execution.
//
// The library links the CUDA runtime statically and reaches the driver only through
// cudaGetDriverEntryPoint, so it loads on a host without a GPU (the CPU test suite checks
// its exports) and needs no libcuda at link time.
#include <cuda.h>
#include <cuda_runtime.h>
#include <nvrtc.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "internal.h"
#include "tgcb.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[2048];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

#define CUDA_TRY(expr)                                                                               \
  do {                                                                                               \
    cudaError_t e_ = (expr);                                                                         \
    if (e_ != cudaSuccess) return fail(TGCB_E_CUDA, "%s failed: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

// Must match struct TgcbArgs in csrc/jit_common.cuh.
struct TgcbArgs {
  char* arena;
  const char* in[TGCB_MAX_INPUTS];
  int* status;
};

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

constexpr int kMaxDevices = kTgcbMaxDevices;
struct DeviceState {
  bool ready = false;
  int* status = nullptr;
  EncodeTiledFn encode = nullptr;
};
DeviceState g_devices[kMaxDevices];
std::mutex g_mutex;

// offset + rows * cols * elem_bytes <= limit, without wrapping around on absurd descriptors
bool fits(uint64_t offset, uint64_t rows, uint64_t cols, uint64_t elem_bytes, uint64_t limit) {
  if (offset > limit) return false;
  const uint64_t room = limit - offset;
  if (elem_bytes == 0 || rows == 0 || cols == 0) return true;
  if (cols > room / elem_bytes) return false;
  const uint64_t row_bytes = cols * elem_bytes;
  return rows <= room / row_bytes;
}

int current_state(DeviceState** out) {
  int dev = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(TGCB_E_INVALID, "device %d out of range", dev);
  if (!g_devices[dev].ready) {
    int rc = tgcb_init(dev);
    if (rc != TGCB_OK) return rc;
  }
  *out = &g_devices[dev];
  return TGCB_OK;
}

}  // namespace

int tgcb_internal_fail(int code, const char* what, const char* detail) { return fail(code, "%s: %s", what, detail); }

int tgcb_internal_status_word(int** out) {
  DeviceState* st = nullptr;
  int rc = current_state(&st);
  if (rc != TGCB_OK) return rc;
  *out = st->status;
  return TGCB_OK;
}

// A loaded module. Its code is context-independent, so plans may run it on any device and
// stream. `done` holds, per device and stream it ran on, an event recorded behind the last
// launches queued there; tgcb_module_unload waits for all of them before releasing the code.
struct tgcb_module {
  struct Done {
    cudaStream_t stream;
    cudaEvent_t event;
  };
  cudaLibrary_t lib = nullptr;
  std::mutex mu;
  std::vector<Done> done[kMaxDevices];
};

struct LaunchState {
  tgcb_launch_desc desc;
  cudaKernel_t kernel = nullptr;
  const void* a_ptr = nullptr;
  const void* b_ptr = nullptr;
  const void* a2_ptr = nullptr;
  const void* b2_ptr = nullptr;
  bool residency_checked = false;  // a chain: every pair can be resident at once
  alignas(64) CUtensorMap ta;
  alignas(64) CUtensorMap tb;
  alignas(64) CUtensorMap ta2;
  alignas(64) CUtensorMap tb2;
};

struct tgcb_plan {
  tgcb_module* module = nullptr;
  std::vector<LaunchState> launches;
  uint64_t arena_bytes = 0;
  int input_count = 0;  // graph inputs the kernels read (tgcb_plan_set_input_count); 0: unchecked
};

extern "C" {

// The NVRTC that compiles generated kernels is whichever libnvrtc.so.12 the process loaded
// first (torch's own copy when torch was imported before this library), so the version string
// names it: the cubin cache is keyed by this string, and a cubin is never reused across NVRTCs.
const char* tgcb_version(void) {
  static std::string version;
  static std::once_flag once;
  std::call_once(once, [] {
    int major = 0, minor = 0;
    char buf[96];
    if (nvrtcVersion(&major, &minor) == NVRTC_SUCCESS)
      snprintf(buf, sizeof(buf), "tgcb 0.2 (sm_100a, nvrtc %d.%d)", major, minor);
    else
      snprintf(buf, sizeof(buf), "tgcb 0.2 (sm_100a, nvrtc unknown)");
    version = buf;
  });
  return version.c_str();
}

const char* tgcb_last_error(void) { return g_last_error.c_str(); }

void tgcb_free(void* p) { free(p); }

int tgcb_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

int tgcb_init(int device) {
  std::lock_guard<std::mutex> lock(g_mutex);
  if (device < 0 || device >= kMaxDevices) return fail(TGCB_E_INVALID, "device %d out of range", device);
  CUDA_TRY(cudaSetDevice(device));
  DeviceState& st = g_devices[device];
  // the allocation-free sum's scratch address, looked up here so its calls need no look-up
  int rc = tgcb_internal_noalloc_setup(device);
  if (rc != TGCB_OK) return rc;
  if (st.ready) return TGCB_OK;
  if (st.status == nullptr) CUDA_TRY(cudaMalloc(reinterpret_cast<void**>(&st.status), 256));  // kept if a later step fails
  CUDA_TRY(cudaMemset(st.status, 0, 256));
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  CUDA_TRY(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
  if (fn == nullptr || q != cudaDriverEntryPointSuccess)
    return fail(TGCB_E_CUDA, "the driver does not provide cuTensorMapEncodeTiled");
  st.encode = reinterpret_cast<EncodeTiledFn>(fn);
  st.ready = true;
  return TGCB_OK;
}

int tgcb_compile_cubin(const char* source, const char* include_dir, const char* const* extra_options,
                       int n_extra_options, void** cubin, size_t* cubin_size, char** log) {
  if (source == nullptr || cubin == nullptr || cubin_size == nullptr)
    return fail(TGCB_E_INVALID, "tgcb_compile_cubin: null argument");
  *cubin = nullptr;
  *cubin_size = 0;
  if (log) *log = nullptr;
  nvrtcProgram prog;
  nvrtcResult r = nvrtcCreateProgram(&prog, source, "tgcb_generated.cu", 0, nullptr, nullptr);
  if (r != NVRTC_SUCCESS) return fail(TGCB_E_COMPILE, "nvrtcCreateProgram: %s", nvrtcGetErrorString(r));
  std::vector<std::string> opts = {"--gpu-architecture=sm_100a", "-std=c++17", "--fmad=false", "-default-device",
                                   "-lineinfo"};
  if (include_dir) opts.push_back(std::string("-I") + include_dir);
  for (int i = 0; i < n_extra_options; ++i) opts.push_back(extra_options[i]);
  std::vector<const char*> copts;
  for (auto& o : opts) copts.push_back(o.c_str());
  r = nvrtcCompileProgram(prog, (int)copts.size(), copts.data());
  size_t log_size = 0;
  nvrtcGetProgramLogSize(prog, &log_size);
  if (log && log_size > 1) {
    *log = static_cast<char*>(malloc(log_size));
    nvrtcGetProgramLog(prog, *log);
  }
  if (r != NVRTC_SUCCESS) {
    nvrtcDestroyProgram(&prog);
    return fail(TGCB_E_COMPILE, "NVRTC could not compile the generated source: %s", nvrtcGetErrorString(r));
  }
  size_t n = 0;
  r = nvrtcGetCUBINSize(prog, &n);
  if (r != NVRTC_SUCCESS || n == 0) {
    nvrtcDestroyProgram(&prog);
    return fail(TGCB_E_COMPILE, "nvrtcGetCUBINSize: %s", nvrtcGetErrorString(r));
  }
  void* buf = malloc(n);
  r = nvrtcGetCUBIN(prog, static_cast<char*>(buf));
  nvrtcDestroyProgram(&prog);
  if (r != NVRTC_SUCCESS) {
    free(buf);
    return fail(TGCB_E_COMPILE, "nvrtcGetCUBIN: %s", nvrtcGetErrorString(r));
  }
  *cubin = buf;
  *cubin_size = n;
  return TGCB_OK;
}

int tgcb_module_load(const void* cubin, size_t size, tgcb_module** out) {
  if (cubin == nullptr || size == 0 || out == nullptr) return fail(TGCB_E_INVALID, "tgcb_module_load: empty image");
  DeviceState* st = nullptr;
  int rc = current_state(&st);
  if (rc != TGCB_OK) return rc;
  auto* m = new tgcb_module();
  cudaError_t e = cudaLibraryLoadData(&m->lib, cubin, nullptr, nullptr, 0, nullptr, nullptr, 0);
  if (e != cudaSuccess) {
    delete m;
    return fail(TGCB_E_CUDA, "cudaLibraryLoadData: %s", cudaGetErrorString(e));
  }
  *out = m;
  return TGCB_OK;
}

int tgcb_module_unload(tgcb_module* m) {
  if (m == nullptr) return TGCB_OK;
  // Kernels of this module queued by the last plan run on each device and stream may still be
  // running: wait for exactly those (not for whole devices), then release the code.
  int rc = TGCB_OK;
  for (int d = 0; d < kMaxDevices; ++d) {
    for (const tgcb_module::Done& x : m->done[d]) {
      cudaError_t e = cudaEventSynchronize(x.event);
      if (e != cudaSuccess && rc == TGCB_OK)
        rc = fail(TGCB_E_CUDA, "waiting for the module's last launches on device %d: %s", d, cudaGetErrorString(e));
      cudaEventDestroy(x.event);
    }
    m->done[d].clear();
  }
  if (rc != TGCB_OK) return rc;  // the code stays loaded: a kernel may still be using it
  if (m->lib) {
    cudaError_t e = cudaLibraryUnload(m->lib);
    if (e != cudaSuccess) rc = fail(TGCB_E_CUDA, "cudaLibraryUnload: %s", cudaGetErrorString(e));
  }
  delete m;
  return rc;
}

int tgcb_plan_create(tgcb_module* m, const tgcb_launch_desc* launches, int n_launches, uint64_t arena_bytes,
                     tgcb_plan** out) {
  if (m == nullptr || out == nullptr || n_launches < 0 || (n_launches > 0 && launches == nullptr))
    return fail(TGCB_E_INVALID, "tgcb_plan_create: bad arguments");
  auto* p = new tgcb_plan();
  p->module = m;
  p->arena_bytes = arena_bytes;
  p->launches.resize(n_launches);
  for (int i = 0; i < n_launches; ++i) {
    LaunchState& ls = p->launches[i];
    ls.desc = launches[i];
    ls.desc.kernel[sizeof(ls.desc.kernel) - 1] = '\0';
    cudaError_t e = cudaLibraryGetKernel(&ls.kernel, m->lib, ls.desc.kernel);
    if (e != cudaSuccess) {
      delete p;
      return fail(TGCB_E_NOT_FOUND, "kernel %s not in module: %s", launches[i].kernel, cudaGetErrorString(e));
    }
    if (ls.desc.smem_bytes > 48 * 1024) {
      e = cudaFuncSetAttribute(reinterpret_cast<const void*>(ls.kernel), cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)ls.desc.smem_bytes);
      if (e != cudaSuccess) {
        delete p;
        return fail(TGCB_E_CUDA, "setting %u bytes of shared memory on %s: %s", ls.desc.smem_bytes, ls.desc.kernel,
                    cudaGetErrorString(e));
      }
    }
    if (ls.desc.is_gemm > 3) {
      delete p;
      return fail(TGCB_E_INVALID, "%s: unknown launch kind %u", ls.desc.kernel, ls.desc.is_gemm);
    }
    const int n_ops = ls.desc.is_gemm == 3 ? 4 : ls.desc.is_gemm ? 2 : 0;
    const tgcb_operand_desc* ops[4] = {&ls.desc.a, &ls.desc.b, &ls.desc.a2, &ls.desc.b2};
    for (int k = 0; k < n_ops; ++k) {
      const tgcb_operand_desc* od = ops[k];
      if (od->input_index >= TGCB_MAX_INPUTS || (od->input_index < 0 && !fits(od->arena_offset, od->rows, od->cols,
                                                                               od->elem_bytes, arena_bytes))) {
        delete p;
        return fail(TGCB_E_INVALID, "operand of %s lies outside the arena or the input table", ls.desc.kernel);
      }
    }
    if ((ls.desc.is_gemm == 3 && ls.desc.counter_bytes == 0) ||
        (ls.desc.counter_bytes > 0 && (!ls.desc.is_gemm || (ls.desc.counter_offset & 3u) != 0 ||
                                       !fits(ls.desc.counter_offset, 1, ls.desc.counter_bytes, 1, arena_bytes)))) {
      delete p;
      return fail(TGCB_E_INVALID, "the counters of %s lie outside the arena", ls.desc.kernel);
    }
  }
  *out = p;
  return TGCB_OK;
}

void tgcb_plan_destroy(tgcb_plan* p) { delete p; }

int tgcb_plan_set_input_count(tgcb_plan* p, int n_inputs) {
  if (p == nullptr) return fail(TGCB_E_INVALID, "tgcb_plan_set_input_count: null plan");
  if (n_inputs < 0 || n_inputs > TGCB_MAX_INPUTS)
    return fail(TGCB_E_INVALID, "a plan reads 0 to %d inputs, not %d", TGCB_MAX_INPUTS, n_inputs);
  p->input_count = n_inputs;
  return TGCB_OK;
}

int tgcb_plan_launch_count(const tgcb_plan* p) { return p ? (int)p->launches.size() : 0; }

static int encode_operand(DeviceState* st, const tgcb_operand_desc& od, const void* base, CUtensorMap* map) {
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return fail(TGCB_E_INVALID, "GEMM operand at %p is not 16-byte aligned", base);
  if ((od.cols * od.elem_bytes) % 16 != 0)
    return fail(TGCB_E_INVALID, "GEMM operand row pitch %llu bytes is not a multiple of 16",
                (unsigned long long)(od.cols * od.elem_bytes));
  CUtensorMapDataType dt = od.elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const CUtensorMapSwizzle sw = od.swizzle == 1 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
  CUresult r;
  if (od.chunks > 0) {
    // 3-D view of the row-major matrix: element (row, 32 q + j) at (j, row, q); one box covers
    // `chunks` consecutive 32-column chunks of box_rows rows, chunk after chunk in shared memory
    if (od.swizzle != 1 || od.elem_bytes != 4 || od.cols % 32 != 0 || od.box_cols != 32 || od.chunks > 8)
      return fail(TGCB_E_INVALID, "a chunked (3-D) operand map needs tf32, the 32-byte-unit swizzle and 32-column chunks");
    cuuint64_t dims[3] = {32, od.rows, od.cols / 32};
    cuuint64_t strides[2] = {od.cols * od.elem_bytes, 32 * od.elem_bytes};
    cuuint32_t box[3] = {32, od.box_rows, od.chunks};
    cuuint32_t estr[3] = {1, 1, 1};
    r = st->encode(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    cuuint64_t dims[2] = {od.cols, od.rows};
    cuuint64_t strides[1] = {od.cols * od.elem_bytes};
    cuuint32_t box[2] = {od.box_cols, od.box_rows};
    cuuint32_t estr[2] = {1, 1};
    r = st->encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) return fail(TGCB_E_CUDA, "cuTensorMapEncodeTiled failed with %d", (int)r);
  return TGCB_OK;
}

}  // extern "C"

namespace {

// Argument checks and the TgcbArgs block shared by every launch of one plan run.
int prepare_run(tgcb_plan* p, void* arena, const void* const* inputs, int n_inputs, DeviceState** st, TgcbArgs* args) {
  if (p == nullptr) return fail(TGCB_E_INVALID, "tgcb_plan_run: null plan");
  if (n_inputs < 0 || n_inputs > TGCB_MAX_INPUTS)
    return fail(TGCB_E_INVALID, "a plan takes at most %d inputs, got %d", TGCB_MAX_INPUTS, n_inputs);
  if (n_inputs > 0 && inputs == nullptr) return fail(TGCB_E_INVALID, "tgcb_plan_run: null input table");
  if (n_inputs < p->input_count)
    return fail(TGCB_E_INVALID, "the plan reads %d inputs, the run passes %d", p->input_count, n_inputs);
  for (int i = 0; i < p->input_count; ++i)
    if (inputs[i] == nullptr) return fail(TGCB_E_INVALID, "input %d of the run is a null pointer", i);
  if (p->arena_bytes > 0 && arena == nullptr) return fail(TGCB_E_INVALID, "tgcb_plan_run: null arena");
  if ((reinterpret_cast<uintptr_t>(arena) & 255u) != 0) return fail(TGCB_E_INVALID, "the arena is not 256-byte aligned");
  int rc = current_state(st);
  if (rc != TGCB_OK) return rc;
  memset(args, 0, sizeof(*args));
  args->arena = static_cast<char*>(arena);
  for (int i = 0; i < n_inputs; ++i) args->in[i] = static_cast<const char*>(inputs[i]);
  args->status = (*st)->status;
  return TGCB_OK;
}

// Queue one launch; GEMM tensor maps are re-encoded only when an operand address changed.
int launch_one(DeviceState* st, LaunchState& ls, TgcbArgs& args, void* arena, const void* const* inputs, int n_inputs,
               cudaStream_t s) {
  const tgcb_launch_desc& d = ls.desc;
  dim3 grid(d.grid[0], d.grid[1], d.grid[2]);
  dim3 block(d.block[0], d.block[1], d.block[2]);
  cudaError_t e;
  if (d.is_gemm) {
    const tgcb_operand_desc* ods[4] = {&d.a, &d.b, &d.a2, &d.b2};
    const void** cached[4] = {&ls.a_ptr, &ls.b_ptr, &ls.a2_ptr, &ls.b2_ptr};
    CUtensorMap* maps[4] = {&ls.ta, &ls.tb, &ls.ta2, &ls.tb2};
    const int n_maps = d.is_gemm == 3 ? 4 : 2;
    for (int k = 0; k < n_maps; ++k) {
      const tgcb_operand_desc& od = *ods[k];
      const void* base;
      if (od.input_index >= 0) {
        if (od.input_index >= n_inputs) return fail(TGCB_E_INVALID, "GEMM operand reads missing input %d", od.input_index);
        base = inputs[od.input_index];
      } else {
        base = static_cast<const char*>(arena) + od.arena_offset;
      }
      if (base != *cached[k]) {
        int rc = encode_operand(st, od, base, maps[k]);
        if (rc != TGCB_OK) return rc;
        *cached[k] = base;
      }
    }
    void* params[5] = {&args, &ls.ta, &ls.tb, &ls.ta2, &ls.tb2};
    if (d.is_gemm >= 2) {
      // two-SM GEMM or chain: clusters of two CTAs (an even grid)
      if ((d.grid[0] & 1u) != 0u) return fail(TGCB_E_INVALID, "%s: a pair GEMM needs an even grid", d.kernel);
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = grid;
      cfg.blockDim = block;
      cfg.dynamicSmemBytes = d.smem_bytes;
      cfg.stream = s;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (d.is_gemm == 3) {
        // A chain's second-GEMM tiles wait for first-GEMM tiles of other pairs, so all pairs
        // must fit on the device together.
        if (!ls.residency_checked) {
          int clusters = 0;
          e = cudaOccupancyMaxActiveClusters(&clusters, reinterpret_cast<const void*>(ls.kernel), &cfg);
          if (e != cudaSuccess) return fail(TGCB_E_CUDA, "cluster occupancy of %s: %s", d.kernel, cudaGetErrorString(e));
          if ((unsigned)clusters < d.grid[0] / 2)
            return fail(TGCB_E_INVALID, "%s needs %u resident SM pairs, the device holds %d", d.kernel, d.grid[0] / 2,
                        clusters);
          ls.residency_checked = true;
        }
      }
      if (d.counter_bytes > 0) {
        // a chain's row-block counters or a K split's region counters start at zero
        e = cudaMemsetAsync(static_cast<char*>(arena) + d.counter_offset, 0, d.counter_bytes, s);
        if (e != cudaSuccess) return fail(TGCB_E_CUDA, "zeroing the counters of %s: %s", d.kernel, cudaGetErrorString(e));
      }
      e = cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(ls.kernel), params);
    } else {
      e = cudaLaunchKernel(reinterpret_cast<const void*>(ls.kernel), grid, block, params, d.smem_bytes, s);
    }
  } else {
    void* params[1] = {&args};
    e = cudaLaunchKernel(reinterpret_cast<const void*>(ls.kernel), grid, block, params, d.smem_bytes, s);
  }
  if (e != cudaSuccess) return fail(TGCB_E_CUDA, "launching %s: %s", d.kernel, cudaGetErrorString(e));
  return TGCB_OK;
}

// Record, behind the launches just queued on `s`, the module's completion event for the current
// device and this stream (created on first use). Inside a stream capture the record becomes a
// node of the graph (cudaEventRecordExternal), so every replay of the graph marks it.
int mark_done(tgcb_module* m, cudaStream_t s) {
  int dev = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(TGCB_E_INVALID, "device %d out of range", dev);
  cudaEvent_t ev = nullptr;
  {
    std::lock_guard<std::mutex> lock(m->mu);
    std::vector<tgcb_module::Done>& list = m->done[dev];
    for (const tgcb_module::Done& x : list)
      if (x.stream == s) ev = x.event;
    if (ev == nullptr) {
      if (list.size() >= 16) {
        // many streams: forget the events whose work has finished
        size_t k = 0;
        for (const tgcb_module::Done& x : list) {
          if (cudaEventQuery(x.event) == cudaSuccess)
            cudaEventDestroy(x.event);
          else
            list[k++] = x;
        }
        list.resize(k);
        cudaGetLastError();  // a query that answered "not ready" leaves that status behind
      }
      CUDA_TRY(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
      list.push_back({s, ev});
    }
  }
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  CUDA_TRY(cudaStreamIsCapturing(s, &cs));
  if (cs == cudaStreamCaptureStatusActive)
    CUDA_TRY(cudaEventRecordWithFlags(ev, s, cudaEventRecordExternal));
  else
    CUDA_TRY(cudaEventRecord(ev, s));
  return TGCB_OK;
}

// Ends a plan run: marks the module's completion on `s` behind whatever was queued, also when a
// launch failed part way (the launches before it are in flight), keeping the first error.
int finish_run(tgcb_plan* p, cudaStream_t s, int rc) {
  if (rc == TGCB_OK) return mark_done(p->module, s);
  const std::string first = g_last_error;
  mark_done(p->module, s);
  g_last_error = first;
  return rc;
}

__global__ void delay_kernel(unsigned long long ns) {
  unsigned long long start;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(start));
  for (int i = 0; i < (1 << 22); ++i) {  // bounded: at most ~4M polls
    unsigned long long now;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
    if (now - start >= ns) break;
    __nanosleep(1000);
  }
}

}  // namespace

extern "C" {

int tgcb_plan_run(tgcb_plan* p, void* arena, const void* const* inputs, int n_inputs, void* stream) {
  DeviceState* st = nullptr;
  TgcbArgs args;
  int rc = prepare_run(p, arena, inputs, n_inputs, &st, &args);
  if (rc != TGCB_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (LaunchState& ls : p->launches) {
    rc = launch_one(st, ls, args, arena, inputs, n_inputs, s);
    if (rc != TGCB_OK) break;
  }
  return finish_run(p, s, rc);
}

int tgcb_plan_run_range(tgcb_plan* p, int first, int count, void* arena, const void* const* inputs, int n_inputs,
                        void* stream) {
  DeviceState* st = nullptr;
  TgcbArgs args;
  int rc = prepare_run(p, arena, inputs, n_inputs, &st, &args);
  if (rc != TGCB_OK) return rc;
  if (first < 0 || count < 0 || (size_t)first + (size_t)count > p->launches.size())
    return fail(TGCB_E_INVALID, "launch range [%d, %d) is outside a plan of %zu launches", first, first + count,
                p->launches.size());
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int i = first; i < first + count; ++i) {
    rc = launch_one(st, p->launches[i], args, arena, inputs, n_inputs, s);
    if (rc != TGCB_OK) break;
  }
  return finish_run(p, s, rc);
}

int tgcb_plan_run_profiled(tgcb_plan* p, void* arena, const void* const* inputs, int n_inputs, void* stream,
                           float* ms) {
  if (ms == nullptr) return fail(TGCB_E_INVALID, "tgcb_plan_run_profiled: null output");
  DeviceState* st = nullptr;
  TgcbArgs args;
  int rc = prepare_run(p, arena, inputs, n_inputs, &st, &args);
  if (rc != TGCB_OK) return rc;
  const size_t n = p->launches.size();
  std::vector<cudaEvent_t> ev(n + 1, nullptr);
  for (auto& e : ev) {
    cudaError_t err = cudaEventCreate(&e);
    if (err != cudaSuccess) {
      rc = fail(TGCB_E_CUDA, "cudaEventCreate: %s", cudaGetErrorString(err));
      break;
    }
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rc == TGCB_OK) {
    cudaError_t err = cudaEventRecord(ev[0], s);
    if (err != cudaSuccess) rc = fail(TGCB_E_CUDA, "cudaEventRecord: %s", cudaGetErrorString(err));
  }
  for (size_t i = 0; i < n && rc == TGCB_OK; ++i) {
    rc = launch_one(st, p->launches[i], args, arena, inputs, n_inputs, s);
    if (rc != TGCB_OK) break;
    cudaError_t err = cudaEventRecord(ev[i + 1], s);
    if (err != cudaSuccess) rc = fail(TGCB_E_CUDA, "cudaEventRecord: %s", cudaGetErrorString(err));
  }
  rc = finish_run(p, s, rc);
  if (rc == TGCB_OK) {
    cudaError_t err = cudaStreamSynchronize(s);
    if (err != cudaSuccess) rc = fail(TGCB_E_CUDA, "cudaStreamSynchronize: %s", cudaGetErrorString(err));
  }
  for (size_t i = 0; i < n && rc == TGCB_OK; ++i) {
    cudaError_t err = cudaEventElapsedTime(&ms[i], ev[i], ev[i + 1]);
    if (err != cudaSuccess) rc = fail(TGCB_E_CUDA, "cudaEventElapsedTime: %s", cudaGetErrorString(err));
  }
  for (auto& e : ev)
    if (e) cudaEventDestroy(e);
  return rc;
}

int tgcb_delay(uint64_t ns, void* stream) {
  if (ns > 10000000ull) ns = 10000000ull;
  delay_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(ns);
  CUDA_TRY(cudaGetLastError());
  return TGCB_OK;
}

int tgcb_status(int clear, int* status) {
  if (status == nullptr) return fail(TGCB_E_INVALID, "tgcb_status: null output");
  DeviceState* st = nullptr;
  int rc = current_state(&st);
  if (rc != TGCB_OK) return rc;
  CUDA_TRY(cudaDeviceSynchronize());
  CUDA_TRY(cudaMemcpy(status, st->status, sizeof(int), cudaMemcpyDeviceToHost));
  if (clear) CUDA_TRY(cudaMemset(st->status, 0, sizeof(int)));
  return TGCB_OK;
}

}  // extern "C"
