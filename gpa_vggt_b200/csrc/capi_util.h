// Host-side helpers shared by the C ABI entry points: error recording, launch
// checks, alignment tests and TMA tensor-map encoding through the driver entry
// point (so the library needs no link-time dependency on libcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdarg.h>
#include <stdio.h>

#include <algorithm>
#include <atomic>
#include <cstring>

#include "../../include/gpa_b200.h"

namespace gpa {

// Last error message of this host thread.
inline char* last_error_buf() {
  static thread_local char buf[512] = {0};
  return buf;
}

inline int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
inline int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(last_error_buf(), 512, fmt, ap);
  va_end(ap);
  return code;
}

inline int ok() { return GPA_OK; }

// Kernels this library has launched in this process (all threads).
inline std::atomic<long long>& launch_counter() {
  static std::atomic<long long> n{0};
  return n;
}

// Record `launched` kernel launches and report a launch error, if any.
inline int check_launch(const char* what, int launched = 1) {
  launch_counter().fetch_add(launched, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(GPA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return GPA_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// cuTensorMapEncodeTiled through cudaGetDriverEntryPoint
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// bf16 tensor map, innermost dim first.  dims/strides_bytes have `rank`
// entries (strides_bytes[0] unused: innermost is contiguous).
inline int make_map_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                         const uint64_t* strides_bytes, const uint32_t* box,
                         CUtensorMapSwizzle swz, const char* what) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return fail(GPA_ERR_CUDA, "%s: cuTensorMapEncodeTiled unavailable", what);
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i > 0) {
      if (strides_bytes[i] % 16)
        return fail(GPA_ERR_INVALID, "%s: stride of dim %d (%llu B) not a multiple of 16", what, i,
                    (unsigned long long)strides_bytes[i]);
      s[i - 1] = strides_bytes[i];
    }
  }
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), d, s, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GPA_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, (int)r);
  return GPA_OK;
}

}  // namespace gpa
