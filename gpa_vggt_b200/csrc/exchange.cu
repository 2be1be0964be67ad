// Merged-block key/value exchange over NVLink peer memory, for the frame-sharded
// forward (one process per GPU, each owning a contiguous range of frames).
//
// Reference: merging/merge.py:234-250 (merge.heads: the scatter-mean of K and V
// into the merged slots) and vggt/layers/attention.py:245-253, which run on one
// device.  Sharded by frames, a merged slot's members sit on several GPUs and
// every GPU's queries need every merged slot.
//
// B200 design.  Each rank keeps its own frames' K/V token rows in a buffer that
// every peer has mapped (CUDA IPC over NVLink/NVSwitch).  One kernel per rank
// walks the output slots whose token lies in its own frames (its dst slots, a
// contiguous ordinal range, and its unmerged src slots): a warp fetches the
// slot's rows -- the kept token, then the members in ascending src ordinal --
// straight from whichever GPU holds them with 16-byte peer loads, sums them in
// fp32 in that fixed order, divides by the count and stores the rounded row
// into the merged buffer of EVERY rank.  So the gather of member rows (an
// all-to-all) and the broadcast of merged rows (an all-gather) happen inside
// the merge itself, tile by tile, and the arithmetic is the one of
// gpa_merge_kv_mean, so the merged rows are bit-identical to one GPU's.  No
// TMA and no multicast: plain loads and stores through peer pointers.
//
// Ordering is the caller's: every rank's row buffer must be complete before any
// rank launches this kernel, and every rank's launch must have finished before
// a merged buffer is read or a row buffer overwritten (the Python side puts a
// one-element NCCL all-reduce on the stream on both sides).
#include "common.cuh"
#include "capi_util.h"

namespace gpa {
namespace xch {

constexpr int kMaxPeers = 8;
constexpr int kThreads = 256;

// 8 elements of a row as raw registers (one 16-byte load for bf16, two for f32)
template <typename T>
struct Raw8;
template <>
struct Raw8<__nv_bfloat16> {
  uint4 a;
  __device__ __forceinline__ void load(const __nv_bfloat16* p) { a = *reinterpret_cast<const uint4*>(p); }
  __device__ __forceinline__ void add_to(float* acc) const {
    const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&a);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(e[i]);
      acc[2 * i] += f.x;
      acc[2 * i + 1] += f.y;
    }
  }
  __device__ __forceinline__ void set(const float* v) {
    __nv_bfloat162* e = reinterpret_cast<__nv_bfloat162*>(&a);
#pragma unroll
    for (int i = 0; i < 4; ++i) e[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  }
  __device__ __forceinline__ void store(__nv_bfloat16* p) const { *reinterpret_cast<uint4*>(p) = a; }
};
template <>
struct Raw8<float> {
  uint4 a, b;
  __device__ __forceinline__ void load(const float* p) {
    a = reinterpret_cast<const uint4*>(p)[0];
    b = reinterpret_cast<const uint4*>(p)[1];
  }
  __device__ __forceinline__ void add_to(float* acc) const {
    acc[0] += __uint_as_float(a.x); acc[1] += __uint_as_float(a.y);
    acc[2] += __uint_as_float(a.z); acc[3] += __uint_as_float(a.w);
    acc[4] += __uint_as_float(b.x); acc[5] += __uint_as_float(b.y);
    acc[6] += __uint_as_float(b.z); acc[7] += __uint_as_float(b.w);
  }
  __device__ __forceinline__ void set(const float* v) {
    a = make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]), __float_as_uint(v[3]));
    b = make_uint4(__float_as_uint(v[4]), __float_as_uint(v[5]), __float_as_uint(v[6]), __float_as_uint(v[7]));
  }
  __device__ __forceinline__ void store(float* p) const {
    reinterpret_cast<uint4*>(p)[0] = a;
    reinterpret_cast<uint4*>(p)[1] = b;
  }
};

// Persistent warps; one work item is a part of an owned slot's row: `split`
// parts of CPL * 256 elements each (lanes take chunks of 8 elements), so a
// 2048-element row is two items and the kernel keeps more warps resident.
// Two rows are in flight per step; the sums still run row by row in the fixed
// order.
template <typename T, int CPL>
__global__ void __launch_bounds__(kThreads) p2p_merge_kernel(
    const T* const* __restrict__ peer_rows, T* const* __restrict__ peer_out, int world, int rank,
    int rows_per_rank, int row_elems, int split, const int32_t* __restrict__ src_pos,
    const int32_t* __restrict__ dst_pos, const int32_t* __restrict__ unm_src, int unm_len,
    const int32_t* __restrict__ seg_start, const int32_t* __restrict__ seg_src, int dst_lo, int dst_hi,
    int* __restrict__ status) {
  const int lane = threadIdx.x & 31;
  const int nch = row_elems / 8;
  const int64_t items = ((int64_t)unm_len + (dst_hi - dst_lo)) * split;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  // a token outside every rank's rows (a malformed plan) reads nothing and
  // flags the status word instead of faulting
  auto row_of = [&](int tok) -> const T* {
    const int o = tok / rows_per_rank;
    if (tok < 0 || o >= world) {
      if (status) atomicOr(status, kDevBadIndex);
      return nullptr;
    }
    return peer_rows[o] + (int64_t)(tok - o * rows_per_rank) * row_elems;
  };

  for (int64_t item = (((int64_t)blockIdx.x * blockDim.x) + threadIdx.x) >> 5; item < items;
       item += nwarps) {
    const int64_t it = item / split;
    const int part = (int)(item - it * split);
    bool live[CPL];
    int ch0[CPL];   // this lane's chunks of the part
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
      ch0[c] = part * 32 * CPL + lane + 32 * c;
      live[c] = ch0[c] < nch;
    }
    int slot, first_tok, s0 = 0, nmem = 0;
    if (it < unm_len) {
      slot = (int)it;
      first_tok = src_pos[unm_src[it]];
      if (first_tok < 0 || first_tok / rows_per_rank != rank) continue;   // another rank's slot
    } else {
      const int d = dst_lo + (int)(it - unm_len);
      slot = unm_len + d;
      first_tok = dst_pos[d];
      s0 = seg_start[d];
      nmem = seg_start[d + 1] - s0;
    }
    float acc[CPL][8];
#pragma unroll
    for (int c = 0; c < CPL; ++c)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[c][i] = 0.0f;
    const int nrows = 1 + nmem;
    for (int b0 = 0; b0 < nrows; b0 += 32) {
      // the batch's token positions, one per lane
      const int nb = min(32, nrows - b0);
      int my_tok = 0;
      if (lane < nb) my_tok = b0 + lane == 0 ? first_tok : src_pos[seg_src[s0 + b0 + lane - 1]];
      for (int i = 0; i < nb; i += 2) {
        const bool two = i + 1 < nb;
        const int ta = __shfl_sync(0xffffffffu, my_tok, i);
        const int tb = __shfl_sync(0xffffffffu, my_tok, two ? i + 1 : i);
        const T* ra = row_of(ta);
        const T* rb = row_of(tb);
        Raw8<T> va[CPL], vb[CPL];
#pragma unroll
        for (int c = 0; c < CPL; ++c)
          if (live[c]) {
            if (ra) va[c].load(ra + ch0[c] * 8);
            if (two && rb) vb[c].load(rb + ch0[c] * 8);
          }
#pragma unroll
        for (int c = 0; c < CPL; ++c)
          if (live[c] && ra) va[c].add_to(acc[c]);
        if (two && rb) {
#pragma unroll
          for (int c = 0; c < CPL; ++c)
            if (live[c]) vb[c].add_to(acc[c]);
        }
      }
    }
    const bool group = slot >= unm_len;
    const float cnt = (float)nrows;
#pragma unroll
    for (int c = 0; c < CPL; ++c)
      if (live[c]) {
        if (group) {
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[c][i] = __fdiv_rn(acc[c][i], cnt);
        }
        Raw8<T> o;
        o.set(acc[c]);
        const int64_t off = (int64_t)slot * row_elems + ch0[c] * 8;
        for (int p = 0; p < world; ++p) o.store(peer_out[p] + off);
      }
  }
  // the stores to peers are performed before the kernel is seen to finish
  __threadfence_system();
}

typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

inline AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(p);
  }
  return fn;
}

}  // namespace xch
}  // namespace gpa

using namespace gpa;
using namespace gpa::xch;

extern "C" int gpa_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  if (!ptr || !handle || !offset) return fail(GPA_ERR_INVALID, "gpa_ipc_export: null pointer");
  AddressRangeFn fn = address_range_fn();
  if (!fn) return fail(GPA_ERR_CUDA, "gpa_ipc_export: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, (CUdeviceptr)ptr) != CUDA_SUCCESS)
    return fail(GPA_ERR_INVALID, "gpa_ipc_export: not a device allocation");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, (void*)base);
  if (e != cudaSuccess) return fail(GPA_ERR_CUDA, "gpa_ipc_export: %s", cudaGetErrorString(e));
  static_assert(sizeof(h) == GPA_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *offset = (int64_t)((uintptr_t)ptr - (uintptr_t)base);
  return ok();
}

extern "C" int gpa_ipc_open(const void* handle, int64_t offset, void** ptr) {
  if (!handle || !ptr || offset < 0) return fail(GPA_ERR_INVALID, "gpa_ipc_open: bad argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(GPA_ERR_CUDA, "gpa_ipc_open: %s", cudaGetErrorString(e));
  *ptr = (void*)((uint8_t*)base + offset);
  return ok();
}

extern "C" int gpa_ipc_close(void* ptr, int64_t offset) {
  if (!ptr || offset < 0) return fail(GPA_ERR_INVALID, "gpa_ipc_close: bad argument");
  cudaError_t e = cudaIpcCloseMemHandle((void*)((uint8_t*)ptr - offset));
  if (e != cudaSuccess) return fail(GPA_ERR_CUDA, "gpa_ipc_close: %s", cudaGetErrorString(e));
  return ok();
}

extern "C" int gpa_merge_exchange_p2p(const void* const* peer_rows, void* const* peer_out, int world,
                                      int rank, int dtype, int rows_per_rank, int row_elems,
                                      const int32_t* src_pos, const int32_t* dst_pos,
                                      const int32_t* unm_src, int unm_len, const int32_t* seg_start,
                                      const int32_t* seg_src, int num_dst, int dst_lo, int dst_hi,
                                      int* status, void* stream) {
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world)
    return fail(GPA_ERR_INVALID, "gpa_merge_exchange_p2p: need 1 <= world <= %d and 0 <= rank < world",
                kMaxPeers);
  if (row_elems <= 0 || row_elems % 8 || row_elems > 8 * 256)
    return fail(GPA_ERR_UNSUPPORTED, "gpa_merge_exchange_p2p: row_elems must be a multiple of 8 up to 2048");
  if (dtype != GPA_DTYPE_BF16 && dtype != GPA_DTYPE_F32)
    return fail(GPA_ERR_INVALID, "gpa_merge_exchange_p2p: dtype must be bf16 or f32");
  if (rows_per_rank <= 0 || unm_len < 0 || num_dst < 0 || dst_lo < 0 || dst_lo > dst_hi || dst_hi > num_dst)
    return fail(GPA_ERR_INVALID, "gpa_merge_exchange_p2p: bad sizes or dst range");
  if (!peer_rows || !peer_out || !src_pos || !dst_pos || (unm_len && !unm_src) || !seg_start ||
      (dst_hi > dst_lo && !seg_src))
    return fail(GPA_ERR_INVALID, "gpa_merge_exchange_p2p: null pointer");
  if (((uintptr_t)peer_rows & 7) || ((uintptr_t)peer_out & 7))
    return fail(GPA_ERR_INVALID, "gpa_merge_exchange_p2p: pointer arrays must be 8-byte aligned");
  const int64_t items = (int64_t)unm_len + (dst_hi - dst_lo);
  if (items == 0) return ok();
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // up to 4 chunks of 8 elements per lane and part (at most 128 registers)
  const int nch = row_elems / 8;
  const int cpl = std::min(4, (nch + 31) / 32);
  const int split = (nch + 32 * cpl - 1) / (32 * cpl);
  const int grid =
      (int)std::min<int64_t>((items * split + kThreads / 32 - 1) / (kThreads / 32), (int64_t)sms * 8);
  cudaStream_t st = (cudaStream_t)stream;
#define GPA_P2P_LAUNCH(T, CPL)                                                                        \
  p2p_merge_kernel<T, CPL><<<grid, kThreads, 0, st>>>(                                              \
      (const T* const*)peer_rows, (T* const*)peer_out, world, rank, rows_per_rank, row_elems, split, \
      src_pos, dst_pos, unm_src, unm_len, seg_start, seg_src, dst_lo, dst_hi, status)
#define GPA_P2P_CPL(T)                                 \
  if (cpl <= 1) GPA_P2P_LAUNCH(T, 1);                  \
  else if (cpl <= 2) GPA_P2P_LAUNCH(T, 2);             \
  else GPA_P2P_LAUNCH(T, 4)
  if (dtype == GPA_DTYPE_BF16) {
    GPA_P2P_CPL(__nv_bfloat16);
  } else {
    GPA_P2P_CPL(float);
  }
#undef GPA_P2P_CPL
#undef GPA_P2P_LAUNCH
  return check_launch("gpa_merge_exchange_p2p");
}
