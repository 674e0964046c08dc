// specq_host.cuh -- host-side plumbing shared by the C-ABI entry points: error reporting,
// per-device state (status word, SM count, kernel attributes), tensor-map encoding through
// the driver entry point (no link-time dependency on libcuda), launch records.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>
#include <string>

#include "specq.h"

namespace specq {

// ---- errors ---------------------------------------------------------------------------------
inline std::string& last_error_ref() {
  static thread_local std::string msg;
  return msg;
}

inline int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  last_error_ref() = buf;
  return code;
}

#define SPECQ_CUDA_TRY(expr)                                                                      \
  do {                                                                                            \
    cudaError_t e_ = (expr);                                                                      \
    if (e_ != cudaSuccess) return ::specq::fail(SPECQ_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

// ---- launch record ----------------------------------------------------------------------------
struct LaunchRecord {
  int variant = -1;
  int grid[3] = {0, 0, 0};
  int cluster_x = 0;
  int threads = 0;
  int dyn_smem = 0;
};
inline LaunchRecord& last_launch_ref() {
  static thread_local LaunchRecord r;
  return r;
}

// ---- per-device state ---------------------------------------------------------------------
constexpr int kMaxDevices = 64;
struct DeviceState {
  bool init = false;
  int sm_count = 0;
  int max_smem_optin = 0;
  int cc_major = 0, cc_minor = 0;
  int* status = nullptr;  // device address of the status word
};

int* device_status_symbol_address();  // defined next to the __device__ status word

inline int get_device_state(DeviceState** out) {
  static std::mutex mu;
  static DeviceState states[kMaxDevices];
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(SPECQ_ERR_NO_DEVICE, "no current CUDA device");
  std::lock_guard<std::mutex> lock(mu);
  DeviceState& st = states[dev];
  if (!st.init) {
    cudaDeviceProp prop;
    SPECQ_CUDA_TRY(cudaGetDeviceProperties(&prop, dev));
    if (prop.major != 10)
      return fail(SPECQ_ERR_NO_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a only", dev,
                  prop.major, prop.minor);
    st.sm_count = prop.multiProcessorCount;
    st.max_smem_optin = static_cast<int>(prop.sharedMemPerBlockOptin);
    st.cc_major = prop.major;
    st.cc_minor = prop.minor;
    st.status = device_status_symbol_address();
    if (st.status == nullptr) return fail(SPECQ_ERR_CUDA, "could not resolve the device status word");
    st.init = true;
  }
  *out = &st;
  return SPECQ_OK;
}

// Raise a kernel's dynamic shared-memory limit once per (kernel, device): the driver call
// otherwise costs about a microsecond of host time on every launch.
inline cudaError_t ensure_dyn_smem(const void* kern, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> granted;
  std::lock_guard<std::mutex> lock(mu);
  int& cur = granted[{kern, dev}];
  if (cur >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) cur = bytes;
  return e;
}

// ---- tensor maps ------------------------------------------------------------------------------
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline PFN_encodeTiled get_encode_tiled() {
  static PFN_encodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  });
  return fn;
}

// Encode a tiled tensor map of rank 2 to 4.  dims/strides_bytes/box are innermost first;
// strides_bytes[i] is the byte stride of dimension i+1.
// Tensor-map encoding is a driver call made several times per operator call; a map depends only
// on its arguments (never on the data), so recently encoded maps are reused from a small
// per-thread table keyed by every argument.
struct TensorMapKey {
  uint64_t words[17];
  bool operator==(const TensorMapKey& o) const { return memcmp(words, o.words, sizeof(words)) == 0; }
};

inline int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                        const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                        CUtensorMapSwizzle swizzle) {
  if (rank < 1 || rank > 5) return fail(SPECQ_ERR_INVALID_ARG, "tensor map of rank %d", rank);
  TensorMapKey key;
  memset(&key, 0, sizeof(key));
  key.words[0] = (static_cast<uint64_t>(dtype) << 32) | (static_cast<uint64_t>(swizzle) << 8) | static_cast<uint64_t>(rank);
  key.words[1] = reinterpret_cast<uint64_t>(base);
  for (int i = 0; i < rank; ++i) {
    key.words[2 + i] = dims[i];
    key.words[7 + i] = box[i];
    if (i + 1 < rank) key.words[12 + i] = strides_bytes[i];
  }
  int dev = -1;
  cudaGetDevice(&dev);
  key.words[16] = static_cast<uint64_t>(static_cast<int64_t>(dev));
  constexpr int kSlots = 64;
  struct Entry {
    TensorMapKey key;
    CUtensorMap map;
    bool valid;
  };
  static thread_local Entry cache[kSlots];
  uint64_t h = 1469598103934665603ull;
  for (uint64_t w : key.words) h = (h ^ w) * 1099511628211ull;
  Entry& slot = cache[(h ^ (h >> 29)) % kSlots];
  if (slot.valid && slot.key == key) {
    *map = slot.map;
    return SPECQ_OK;
  }
  PFN_encodeTiled enc = get_encode_tiled();
  if (enc == nullptr) return fail(SPECQ_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  CUresult r = enc(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, s, b, e,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SPECQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
  slot.key = key;
  slot.map = *map;
  slot.valid = true;
  return SPECQ_OK;
}

// ---- small integer helpers --------------------------------------------------------------------
inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
inline int round_up(int a, int b) { return ceil_div(a, b) * b; }
inline int next_pow2(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}
inline bool aligned(const void* p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

// Programmatic dependent launch: every kernel of this library may be scheduled while the
// previous kernel on its stream is still finishing (its CTAs then wait in griddepcontrol.wait
// before touching global memory), which hides the launch latency between back-to-back kernels.
// SPECQ_PDL=0 in the environment turns it off.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("SPECQ_PDL");
    return v == nullptr || v[0] != '0';
  }();
  return on;
}

// Launch attributes: the cluster shape (when > 1) and programmatic dependent launch.
struct LaunchAttrs {
  cudaLaunchAttribute a[2];
  unsigned n = 0;
  explicit LaunchAttrs(int cluster_x) {
    if (cluster_x > 1) {
      a[n].id = cudaLaunchAttributeClusterDimension;
      a[n].val.clusterDim.x = static_cast<unsigned>(cluster_x);
      a[n].val.clusterDim.y = 1;
      a[n].val.clusterDim.z = 1;
      ++n;
    }
    if (pdl_enabled()) {
      a[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      a[n].val.programmaticStreamSerializationAllowed = 1;
      ++n;
    }
  }
  void apply(cudaLaunchConfig_t& cfg) {
    cfg.attrs = a;
    cfg.numAttrs = n;
  }
};

// cudaLaunchKernelEx with the library's launch attributes and no cluster.
template <typename... Params, typename... Args>
inline cudaError_t launch_plain(void (*kern)(Params...), dim3 grid, dim3 block, cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  LaunchAttrs at(1);
  at.apply(cfg);
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Widest access width (16, 8, 4, 2, 1 bytes) that every pointer and byte count in the list
// is a multiple of.
inline int common_vec_width(std::initializer_list<uint64_t> values) {
  int w = 16;
  for (uint64_t v : values) {
    while (w > 1 && (v % static_cast<uint64_t>(w)) != 0) w >>= 1;
  }
  return w;
}

}  // namespace specq
