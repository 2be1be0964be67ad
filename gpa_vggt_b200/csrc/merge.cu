// Bipartite K/V token merging on B200: dst/src roles, projected-metric
// normalisation + split, the merge plan (top-r selection, per-dst groups,
// counts) and the deterministic scatter-mean of K/V.
//
// Reference algorithm: merging/merge.py:39-256 (token_merge_bipartite2d).
// All of it is integer/byte work or HBM-bound streaming; nothing here is a
// GEMM.  Differences of representation (not of result):
//  * dst and src are enumerated in ascending token position (the reference's
//    argsort of the -1/0 mask, merge.py:165, is unstable; any order of the
//    same sets gives the same attention output since the slots only permute).
//  * the top-r edge selection breaks ties at the cut by src ordinal (a stable
//    descending sort); merge.py:199 uses an unstable argsort.
//  * group sums run in fp32 in a fixed order (dst, then src ordinal
//    ascending), so results are deterministic, unlike scatter_reduce's atomics.
#include "common.cuh"
#include "capi_util.h"

namespace gpa {

// ---------------------------------------------------------------------------
// roles (merging/merge.py:87-176)
// ---------------------------------------------------------------------------
struct RoleGeom {
  int P, w, h, sx, sy, ns, no_rand;
  int hsy, wsx, eh, ew, dpf;  // dst per frame for f >= 1
};

__device__ __forceinline__ bool token_is_dst(const RoleGeom& g, const int64_t* rand_idx, int f,
                                             int p) {
  if (f == 0 || p < g.ns) return true;
  if (g.no_rand) return false;  // merge.py:105-118 writes 0 (src) on the whole grid
  int q = p - g.ns;
  if (q >= g.eh * g.ew) return false;  // trailing patch tokens are always src
  int row = q / g.ew, col = q - row * g.ew;
  int wy = row / g.sy, dy = row - wy * g.sy;
  int wx = col / g.sx, dx = col - wx * g.sx;
  int64_t pick = rand_idx[((int64_t)(f - 1) * g.hsy + wy) * g.wsx + wx];
  return pick == (int64_t)(dy * g.sx + dx);
}

// one block per frame, ordinals by a block-wide scan over the frame's tokens
template <int THREADS>
__global__ void __launch_bounds__(THREADS) roles_kernel(RoleGeom g, const int64_t* rand_idx,
                                                         int32_t* dst_pos, int32_t* src_pos,
                                                         int32_t* slot) {
  const int f = blockIdx.x;
  const int per = (g.P + THREADS - 1) / THREADS;
  const int p0 = threadIdx.x * per;
  const int p1 = min(p0 + per, g.P);
  int nd = 0;
  for (int p = p0; p < p1; ++p) nd += token_is_dst(g, rand_idx, f, p) ? 1 : 0;

  // block exclusive scan of nd
  __shared__ int warp_tot[THREADS / 32];
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int incl = nd;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) warp_tot[wid] = incl;
  __syncthreads();
  if (wid == 0) {
    int v = lane < THREADS / 32 ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int t = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += t;
    }
    if (lane < THREADS / 32) warp_tot[lane] = v;  // inclusive
  }
  __syncthreads();
  int dst_rank = incl - nd + (wid > 0 ? warp_tot[wid - 1] : 0);
  int src_rank = p0 - dst_rank;

  const int64_t fbase = (int64_t)f * g.P;
  const int64_t dst_base = f == 0 ? 0 : (int64_t)g.P + (int64_t)(f - 1) * g.dpf;
  const int64_t src_base = f == 0 ? 0 : (int64_t)(f - 1) * (g.P - g.dpf);
  for (int p = p0; p < p1; ++p) {
    int64_t pos = fbase + p;
    if (token_is_dst(g, rand_idx, f, p)) {
      int64_t o = dst_base + dst_rank++;
      dst_pos[o] = (int32_t)pos;
      slot[pos] = (int32_t)o;
    } else {
      int64_t o = src_base + src_rank++;
      src_pos[o] = (int32_t)pos;
      slot[pos] = (int32_t)(-o - 1);
    }
  }
}

template <typename T>
struct Vec8;
template <>
struct Vec8<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float* v) {
    uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
    const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(e[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
  static __device__ __forceinline__ void load_shared(const __nv_bfloat16* p, float* v) {
    uint4 raw = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(e[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float* v) {
    uint4 raw;
    __nv_bfloat162* e = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) e[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = raw;
  }
};
template <>
struct Vec8<float> {
  static __device__ __forceinline__ void load(const float* p, float* v) {
    float4 a = __ldg(reinterpret_cast<const float4*>(p));
    float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  static __device__ __forceinline__ void load_shared(const float* p, float* v) {
    float4 a = reinterpret_cast<const float4*>(p)[0];
    float4 b = reinterpret_cast<const float4*>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  static __device__ __forceinline__ void store(float* p, const float* v) {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
};

// ---------------------------------------------------------------------------
// metric normalise + split (merging/merge.py:185-187)
// ---------------------------------------------------------------------------
// one warp per output row; rows < num_src go to a, the rest to b
template <typename T>
__global__ void metric_split_kernel(const T* __restrict__ metric, int64_t stride,
                                    int d, const int32_t* __restrict__ src_pos, int num_src,
                                    const int32_t* __restrict__ dst_pos, int num_dst,
                                    __nv_bfloat16* __restrict__ a, __nv_bfloat16* __restrict__ b) {
  int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (row >= num_src + num_dst) return;
  int tok;
  __nv_bfloat16* out;
  if (row < num_src) {
    tok = src_pos[row];
    out = a + (int64_t)row * d;
  } else {
    tok = dst_pos[row - num_src];
    out = b + (int64_t)(row - num_src) * d;
  }
  const T* in = metric + (int64_t)tok * stride;
  // d <= 1024: up to 4 chunks of 8 per lane
  float v[4][8];
  float ss = 0.f;
  const int nch = d / 8;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    int ch = lane + c * 32;
    if (ch < nch) {
      Vec8<T>::load(in + ch * 8, v[c]);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(v[c][i], v[c][i], ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  // fp32 norm and quotient, rounded to bf16 once: the reference's GPU run under
  // autocast computes `metric.norm()` in fp32 (norm is on autocast's fp32
  // list), so `metric / norm` is an fp32 division even for a bf16 metric, and
  // the matcher casts the quotient to bf16 (fused_similarity.py:99-101)
  float nrm = __fsqrt_rn(ss);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    int ch = lane + c * 32;
    if (ch < nch) {
      uint4 raw;
      __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&raw);
#pragma unroll
      for (int i = 0; i < 8; ++i) e[i] = __float2bfloat16_rn(__fdiv_rn(v[c][i], nrm));
      *reinterpret_cast<uint4*>(out + ch * 8) = raw;
    }
  }
}

// ---------------------------------------------------------------------------
// device-wide exclusive scan of int32 (n <= 1024*1024), 3 launches
// ---------------------------------------------------------------------------
constexpr int kScanBlock = 1024;  // elements per block (256 threads x 4)

__device__ __forceinline__ int block_excl_scan_256(int v, int* total) {
  __shared__ int wsum[8];
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) wsum[wid] = incl;
  __syncthreads();
  if (wid == 0) {
    int w = lane < 8 ? wsum[lane] : 0;
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      int t = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += t;
    }
    if (lane < 8) wsum[lane] = w;
  }
  __syncthreads();
  int res = incl - v + (wid > 0 ? wsum[wid - 1] : 0);
  if (total) *total = wsum[7];
  __syncthreads();
  return res;
}

// MODE 0: scan in[]; MODE 1: scan of (in[i] == 0)
template <int MODE>
__global__ void __launch_bounds__(256) scan_local_kernel(const int* __restrict__ in,
                                                         int* __restrict__ out, int n,
                                                         int* __restrict__ block_sums) {
  int base = blockIdx.x * kScanBlock + threadIdx.x * 4;
  int v[4];
  int s = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int x = base + i < n ? in[base + i] : 0;
    if (MODE == 1) x = (base + i < n) ? (x == 0 ? 1 : 0) : 0;
    v[i] = x;
    s += x;
  }
  int tot;
  int ex = block_excl_scan_256(s, &tot);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (base + i < n) out[base + i] = ex;
    ex += v[i];
  }
  if (threadIdx.x == 0) block_sums[blockIdx.x] = tot;
}

__global__ void __launch_bounds__(1024) scan_blocks_kernel(int* __restrict__ block_sums, int nb,
                                                           int* __restrict__ total_out) {
  __shared__ int wsum[32];
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int v = threadIdx.x < nb ? block_sums[threadIdx.x] : 0;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) wsum[wid] = incl;
  __syncthreads();
  if (wid == 0) {
    int w = wsum[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int t = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += t;
    }
    wsum[lane] = w;
  }
  __syncthreads();
  int ex = incl - v + (wid > 0 ? wsum[wid - 1] : 0);
  if (threadIdx.x < nb) block_sums[threadIdx.x] = ex;
  if (threadIdx.x == 0 && total_out) *total_out = wsum[31];
}

__global__ void scan_add_kernel(int* __restrict__ out, int n, const int* __restrict__ block_sums) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] += block_sums[i / kScanBlock];
}

template <int MODE>
static int exclusive_scan(const int* in, int* out, int n, int* block_sums, int* total,
                          cudaStream_t st) {
  int nb = (n + kScanBlock - 1) / kScanBlock;
  if (nb == 0) nb = 1;
  scan_local_kernel<MODE><<<nb, 256, 0, st>>>(in, out, n, block_sums);
  scan_blocks_kernel<<<1, 1024, 0, st>>>(block_sums, nb, total);
  if (n > 0) scan_add_kernel<<<(n + 255) / 256, 256, 0, st>>>(out, n, block_sums);
  return n > 0 ? 3 : 2;
}

// ---------------------------------------------------------------------------
// merge plan (merging/merge.py:189-217)
// ---------------------------------------------------------------------------
// order-preserving map float -> uint32 (ascending)
__device__ __forceinline__ uint32_t float_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

struct SelectState {
  uint32_t prefix;     // high bits of the threshold key found so far
  uint32_t remaining;  // how many of the top elements are still to be taken
};

constexpr int kRadixPasses = 3;
__host__ __device__ constexpr int radix_shift(int pass) { return pass == 0 ? 21 : (pass == 1 ? 10 : 0); }
__host__ __device__ constexpr int radix_bits(int pass) { return pass == 2 ? 10 : 11; }

__global__ void select_hist_kernel(const float* __restrict__ node_max, int n, int pass,
                                   const SelectState* __restrict__ st, unsigned* __restrict__ hist) {
  __shared__ unsigned sh[2048];
  for (int i = threadIdx.x; i < 2048; i += blockDim.x) sh[i] = 0;
  __syncthreads();
  const int shift = radix_shift(pass), bits = radix_bits(pass);
  const uint32_t hi_shift = shift + bits;
  const uint32_t prefix = st->prefix;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    uint32_t k = float_key(node_max[i]);
    bool match = (hi_shift >= 32) ? true : ((k >> hi_shift) == (prefix >> hi_shift));
    if (match) atomicAdd(&sh[(k >> shift) & ((1u << bits) - 1)], 1u);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < (1 << bits); i += blockDim.x)
    if (sh[i]) atomicAdd(&hist[i], sh[i]);
}

// threshold state {prefix 0, r still to take} and a zeroed histogram, written on
// the device so the plan issues no host-to-device copy
__global__ void select_init_kernel(SelectState* st, unsigned* hist, uint32_t r) {
  for (int i = threadIdx.x; i < 2048; i += blockDim.x) hist[i] = 0u;
  if (threadIdx.x == 0) {
    st->prefix = 0u;
    st->remaining = r;
  }
}

// single thread: walk the histogram from the top bin down
__global__ void select_pick_kernel(int pass, SelectState* st, unsigned* hist) {
  const int shift = radix_shift(pass), bits = radix_bits(pass);
  uint32_t rem = st->remaining;
  int b = (1 << bits) - 1;
  for (; b > 0; --b) {
    uint32_t c = hist[b];
    if (c >= rem) break;
    rem -= c;
  }
  st->prefix |= ((uint32_t)b) << shift;
  st->remaining = rem;
  for (int i = 0; i < (1 << bits); ++i) hist[i] = 0;
}

// flags[i] = 1 if src i is merged; eq[i] = 1 if key == threshold (ties at the cut)
__global__ void select_flags_kernel(const float* __restrict__ node_max, int n,
                                    const SelectState* __restrict__ st, int* __restrict__ gt,
                                    int* __restrict__ eq) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  uint32_t k = float_key(node_max[i]);
  gt[i] = k > st->prefix ? 1 : 0;
  eq[i] = k == st->prefix ? 1 : 0;
}

// merged = gt || (eq && rank among eq < remaining);  writes merged flag into gt
__global__ void select_final_kernel(int n, const SelectState* __restrict__ st, int* __restrict__ gt,
                                    const int* __restrict__ eq, const int* __restrict__ eq_rank) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  if (!gt[i] && eq[i] && eq_rank[i] < (int)st->remaining) gt[i] = 1;
}

__global__ void fill_ones_kernel(int* __restrict__ f, int n) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) f[i] = 1;
}

__global__ void group_hist_kernel(const int32_t* __restrict__ node_idx, const int* __restrict__ merged,
                                  int n, int* __restrict__ seg_len) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n && merged[i]) atomicAdd(&seg_len[node_idx[i]], 1);
}

// merged src, in ascending ordinal, go to their merged rank as (key = dst
// ordinal, value = src ordinal); unmerged src go to unm_src at their unmerged
// rank, which is the ordinal minus the merged rank
__global__ void group_compact_kernel(const int32_t* __restrict__ node_idx, const int* __restrict__ merged,
                                     const int* __restrict__ mrank, int n, int32_t* __restrict__ keys,
                                     int32_t* __restrict__ vals, int32_t* __restrict__ unm_src) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int at = mrank[i];
  if (merged[i]) {
    if (keys) keys[at] = node_idx[i];
    vals[at] = i;
  } else {
    unm_src[i - at] = i;
  }
}

// Stable LSD radix sort of the merged (dst, src) pairs by dst, 8 bits a pass:
// a group's members come out in ascending src ordinal without atomics, in time
// linear in the number of merged src whatever the group sizes.
constexpr int kRadixItems = 1024;   // pairs per block of one pass
constexpr int kRadixDigits = 256;

// per block: how many of its pairs fall in each digit -> table[digit][block]
__global__ void __launch_bounds__(kRadixDigits) radix_hist_kernel(const int32_t* __restrict__ keys, int n,
                                                                   int shift, int nblk, int* __restrict__ table) {
  __shared__ int h[kRadixDigits];
  h[threadIdx.x] = 0;
  __syncthreads();
  const int b0 = blockIdx.x * kRadixItems;
  for (int k = threadIdx.x; k < kRadixItems; k += kRadixDigits) {
    const int i = b0 + k;
    if (i < n) atomicAdd(&h[(keys[i] >> shift) & (kRadixDigits - 1)], 1);
  }
  __syncthreads();
  table[threadIdx.x * nblk + blockIdx.x] = h[threadIdx.x];
}

// one warp per block of pairs, 32 at a time in pair order, so equal digits keep
// their order: lanes with one digit share the digit's running offset and take
// their rank among themselves; the lowest of them advances the offset
__global__ void __launch_bounds__(32) radix_scatter_kernel(const int32_t* __restrict__ kin,
                                                           const int32_t* __restrict__ vin, int n, int shift,
                                                           int nblk, const int* __restrict__ offsets,
                                                           int32_t* __restrict__ kout, int32_t* __restrict__ vout) {
  __shared__ int base[kRadixDigits];
  const int lane = threadIdx.x;
  for (int d = lane; d < kRadixDigits; d += 32) base[d] = offsets[d * nblk + blockIdx.x];
  __syncwarp();
  const int b0 = blockIdx.x * kRadixItems;
  for (int c = 0; c < kRadixItems && b0 + c < n; c += 32) {   // warp-uniform
    const int i = b0 + c + lane;
    const bool live = i < n;
    const int key = live ? kin[i] : 0;
    const int val = live ? vin[i] : 0;
    const int d = live ? (key >> shift) & (kRadixDigits - 1) : kRadixDigits + lane;
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    const int pos = live ? base[d] + rank : 0;
    __syncwarp();
    if (live && rank == 0) base[d] += __popc(peers);
    __syncwarp();
    if (live) {
      if (kout) kout[pos] = key;
      vout[pos] = val;
    }
  }
}

// counts of the dst slots: 1 + group size
__global__ void group_counts_kernel(const int32_t* __restrict__ seg_start, int num_dst,
                                    float* __restrict__ counts, int unm_len) {
  int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g < num_dst) counts[unm_len + g] = (float)(1 + seg_start[g + 1] - seg_start[g]);
}

__global__ void ones_f32_kernel(float* __restrict__ f, int n) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) f[i] = 1.0f;
}

// ---------------------------------------------------------------------------
// scatter-mean (merging/merge.py:234-250)
// ---------------------------------------------------------------------------
// One warp per output slot; the warp's lanes cover heads*head_dim in chunks of
// 8 elements, up to CPL chunks per lane (heads*head_dim <= CPL*256).
//
// The group's rows (the dst token first, then its src members in ascending
// ordinal order) are fetched ROWS at a time with cp.async into this warp's
// shared-memory staging area: the token positions of a batch are resolved one
// per lane in parallel, and every row copy of the batch is in flight at once
// without holding registers.  Warps are persistent and double-buffer their
// batches, so the index loads and row copies of the next batch overlap the
// wait for this one.  The fp32 sums run in the fixed row order
// (deterministic, unlike the reference's scatter_reduce).
#ifndef GPA_MERGE_WARPS
#define GPA_MERGE_WARPS 2
#endif
#ifndef GPA_MERGE_ROWS
#define GPA_MERGE_ROWS 2
#endif
constexpr int kMergeWarps = GPA_MERGE_WARPS;   // warps (persistent slot walkers) per block
constexpr int kMergeRows = GPA_MERGE_ROWS;     // rows per staged batch (two batches per warp)

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// One batch of a slot's rows: the slot, its kept token, its members and which
// ROWS-row batch of them.
struct MergeItem {
  int slot, first_tok, s0, nmem, batch;
};

template <typename T, int CPL>
__global__ void __launch_bounds__(kMergeWarps * 32) merge_mean_kernel(
    const T* __restrict__ t, int heads, int head_dim, int64_t sh, int64_t sn,
    const int32_t* __restrict__ src_pos, const int32_t* __restrict__ dst_pos,
    const int32_t* __restrict__ unm_src, int unm_len, const int32_t* __restrict__ seg_start,
    const int32_t* __restrict__ seg_src, int num_dst, int reduce_mean,
    float* __restrict__ log_counts, T* __restrict__ out, int64_t osh, int64_t osn, int rows_per_batch) {
  extern __shared__ __align__(16) uint8_t merge_smem[];
  constexpr int kChunk = 8 * (int)sizeof(T);       // bytes of 8 elements
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slots = unm_len + num_dst;
  const int warps_total = gridDim.x * kMergeWarps;
  const int first_slot = blockIdx.x * kMergeWarps + warp;
  if (first_slot >= slots) return;                 // warp-uniform
  const int cph = head_dim / 8;        // chunks per head
  const int nch = heads * cph;         // chunks per token
  int64_t in_off[CPL], out_off[CPL];
  bool live[CPL];
#pragma unroll
  for (int c = 0; c < CPL; ++c) {
    int ch = lane + c * 32;
    live[c] = ch < nch;
    int hh = live[c] ? ch / cph : 0;
    int d0 = live[c] ? (ch - hh * cph) * 8 : 0;
    in_off[c] = (int64_t)hh * sh + d0;
    out_off[c] = (int64_t)hh * osh + d0;
  }
  const size_t stage_bytes = (size_t)rows_per_batch * nch * kChunk;
  uint8_t* stages = merge_smem + (size_t)warp * 2 * stage_bytes;

  auto load_slot = [&](int sl, MergeItem& it) {
    it.slot = sl;
    it.batch = 0;
    if (sl < unm_len) {
      it.first_tok = src_pos[unm_src[sl]];
      it.s0 = 0;
      it.nmem = 0;
    } else {
      const int g = sl - unm_len;
      it.first_tok = dst_pos[g];
      it.s0 = seg_start[g];
      it.nmem = seg_start[g + 1] - it.s0;
    }
  };
  // the next batch of the same slot, else the first batch of this warp's next slot
  auto advance = [&](MergeItem& it) -> bool {
    if ((it.batch + 1) * rows_per_batch < 1 + it.nmem) {
      ++it.batch;
      return true;
    }
    const int ns = it.slot + warps_total;
    if (ns >= slots) return false;
    load_slot(ns, it);
    return true;
  };
  // resolve the batch's token positions (one per lane) and start its row copies
  auto issue = [&](const MergeItem& it, uint8_t* stage) {
    const int base = it.batch * rows_per_batch;
    const int nb = min(rows_per_batch, 1 + it.nmem - base);
    int my_tok = 0;
    if (lane < nb) my_tok = base + lane == 0 ? it.first_tok : src_pos[seg_src[it.s0 + base + lane - 1]];
    for (int i = 0; i < nb; ++i) {
      const int64_t tok = __shfl_sync(0xffffffffu, my_tok, i);
      const uint8_t* row = reinterpret_cast<const uint8_t*>(t + tok * sn);
#pragma unroll
      for (int c = 0; c < CPL; ++c)
        if (live[c]) {
          uint8_t* dst = stage + ((size_t)i * nch + lane + c * 32) * kChunk;
          const uint8_t* src = row + in_off[c] * (int64_t)sizeof(T);
#pragma unroll
          for (int q = 0; q < kChunk / 16; ++q) cp_async16(dst + q * 16, src + q * 16);
        }
    }
    cp_async_commit();
  };

  float acc[CPL][8];
#pragma unroll
  for (int c = 0; c < CPL; ++c)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[c][i] = 0.0f;
  MergeItem cur;
  load_slot(first_slot, cur);
  issue(cur, stages);
  int buf = 0;
  while (true) {
    // the next batch's index loads and row copies overlap this batch's wait
    MergeItem nxt = cur;
    const bool more = advance(nxt);
    if (more) {
      issue(nxt, stages + (buf ^ 1) * stage_bytes);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    // each lane reads back only the chunks it copied
    const uint8_t* stage = stages + buf * stage_bytes;
    const int nb = min(rows_per_batch, 1 + cur.nmem - cur.batch * rows_per_batch);
    for (int i = 0; i < nb; ++i) {
#pragma unroll
      for (int c = 0; c < CPL; ++c)
        if (live[c]) {
          float v[8];
          Vec8<T>::load_shared(reinterpret_cast<const T*>(stage + ((size_t)i * nch + lane + c * 32) * kChunk), v);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[c][e] += v[e];
        }
    }
    if ((cur.batch + 1) * rows_per_batch >= 1 + cur.nmem) {   // the slot's last batch
      const bool group = cur.slot >= unm_len;
      const float cnt = (float)(1 + cur.nmem);
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        if (live[c]) {
          if (group && reduce_mean) {
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[c][i] = __fdiv_rn(acc[c][i], cnt);
          }
          Vec8<T>::store(out + out_off[c] + (int64_t)cur.slot * osn, acc[c]);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[c][i] = 0.0f;
      }
      if (log_counts && lane == 0) log_counts[cur.slot] = group ? logf(cnt) : 0.0f;
    }
    if (!more) break;
    cur = nxt;
    buf ^= 1;
  }
}

}  // namespace gpa

using namespace gpa;

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" int gpa_merge_counts(int num_imgs, int w, int h, int sx, int sy, int num_special,
                                int no_rand, int* num_dst, int* num_src) {
  if (num_imgs < 0 || w <= 0 || h <= 0 || sx <= 0 || sy <= 0 || num_special < 0 || !num_dst ||
      !num_src)
    return fail(GPA_ERR_INVALID, "gpa_merge_counts: bad geometry");
  const int64_t P = (int64_t)w * h + num_special;
  const int64_t N = P * num_imgs;
  if (N >= (1ll << 31)) return fail(GPA_ERR_UNSUPPORTED, "gpa_merge_counts: too many tokens");
  const int64_t dpf = num_special + (no_rand ? 0 : (int64_t)(h / sy) * (w / sx));
  const int64_t nd = num_imgs > 0 ? P + (int64_t)(num_imgs - 1) * dpf : 0;
  *num_dst = (int)nd;
  *num_src = (int)(N - nd);
  return ok();
}

extern "C" int gpa_merge_roles(const int64_t* rand_idx, int num_imgs, int w, int h, int sx, int sy,
                               int num_special, int no_rand, int32_t* dst_pos, int32_t* src_pos,
                               int32_t* slot, void* stream) {
  int nd, ns;
  int rc = gpa_merge_counts(num_imgs, w, h, sx, sy, num_special, no_rand, &nd, &ns);
  if (rc) return rc;
  if (num_imgs == 0) return ok();
  if (!dst_pos || !slot || (ns > 0 && !src_pos) || (!no_rand && num_imgs > 1 && !rand_idx))
    return fail(GPA_ERR_INVALID, "gpa_merge_roles: null pointer");
  RoleGeom g;
  g.P = w * h + num_special;
  g.w = w; g.h = h; g.sx = sx; g.sy = sy; g.ns = num_special; g.no_rand = no_rand;
  g.hsy = h / sy; g.wsx = w / sx;
  g.eh = g.hsy * sy; g.ew = g.wsx * sx;
  g.dpf = num_special + (no_rand ? 0 : g.hsy * g.wsx);
  roles_kernel<256><<<num_imgs, 256, 0, (cudaStream_t)stream>>>(g, rand_idx, dst_pos, src_pos, slot);
  return check_launch("gpa_merge_roles");
}

extern "C" int gpa_metric_split(const void* metric, int dtype, int64_t metric_stride, int d,
                                const int32_t* src_pos, int num_src, const int32_t* dst_pos,
                                int num_dst, void* a, void* b, void* stream) {
  if (d <= 0 || d % 8 || d > 1024 || metric_stride % 8 || num_src < 0 || num_dst < 0)
    return fail(GPA_ERR_INVALID, "gpa_metric_split: need d %% 8 == 0, d <= 1024, stride %% 8 == 0");
  if (!aligned16(metric) || (num_src && !aligned16(a)) || (num_dst && !aligned16(b)))
    return fail(GPA_ERR_INVALID, "gpa_metric_split: pointers must be 16-byte aligned");
  if (dtype != GPA_DTYPE_F32 && dtype != GPA_DTYPE_BF16)
    return fail(GPA_ERR_INVALID, "gpa_metric_split: dtype must be f32 or bf16");
  int rows = num_src + num_dst;
  if (rows == 0) return ok();
  if (dtype == GPA_DTYPE_BF16)
    metric_split_kernel<__nv_bfloat16><<<(rows + 7) / 8, 256, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16*)metric, metric_stride, d, src_pos, num_src, dst_pos, num_dst,
        (__nv_bfloat16*)a, (__nv_bfloat16*)b);
  else
    metric_split_kernel<float><<<(rows + 7) / 8, 256, 0, (cudaStream_t)stream>>>(
        (const float*)metric, metric_stride, d, src_pos, num_src, dst_pos, num_dst,
        (__nv_bfloat16*)a, (__nv_bfloat16*)b);
  return check_launch("gpa_metric_split");
}

// workspace layout (int32 words unless noted)
namespace {
struct PlanWs {
  SelectState* st;
  unsigned* hist;
  int* block_sums;
  int* flags;    // merged
  int* eq;       // tie flags; later the radix sort's second key buffer
  int* rank;     // rank among the ties, then merged rank
  int* seg_len;  // per dst
  int32_t* key_a;
  int32_t* val_a;
  int32_t* val_b;
  int* table;    // radix digit x block counts, then their offsets
};
int radix_blocks(int n) { return (n + kRadixItems - 1) / kRadixItems; }
int64_t plan_ws_layout(int num_src, int num_dst, char* base, PlanWs* w) {
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    char* p = base ? base + off : nullptr;
    off += (bytes + 255) & ~int64_t(255);
    return p;
  };
  const int64_t table = (int64_t)kRadixDigits * std::max(1, radix_blocks(num_src));
  const int64_t scanned = std::max<int64_t>(std::max(num_src, num_dst + 1), table);
  const int64_t nblk = (scanned + kScanBlock - 1) / kScanBlock + 1;
  PlanWs t;
  t.st = (SelectState*)take(sizeof(SelectState) * 2);
  t.hist = (unsigned*)take(2048 * 4);
  t.block_sums = (int*)take(nblk * 4);
  t.flags = (int*)take((int64_t)num_src * 4);
  t.eq = (int*)take((int64_t)num_src * 4);
  t.rank = (int*)take((int64_t)num_src * 4);
  t.seg_len = (int*)take((int64_t)(num_dst + 1) * 4);
  t.key_a = (int32_t*)take((int64_t)num_src * 4);
  t.val_a = (int32_t*)take((int64_t)num_src * 4);
  t.val_b = (int32_t*)take((int64_t)num_src * 4);
  t.table = (int*)take(table * 4);
  if (w) *w = t;
  return off;
}
}  // namespace

extern "C" int64_t gpa_merge_plan_workspace_bytes(int num_src, int num_dst) {
  if (num_src < 0 || num_dst < 0) return -1;
  return plan_ws_layout(num_src, num_dst, nullptr, nullptr);
}

extern "C" int gpa_merge_plan(const float* node_max, const int32_t* node_idx, int num_src,
                              int num_dst, int r, int32_t* unm_src, int32_t* seg_start,
                              int32_t* seg_src, float* counts, void* workspace,
                              int64_t workspace_bytes, void* stream) {
  if (num_src < 0 || num_dst <= 0 || r < 0)
    return fail(GPA_ERR_INVALID, "gpa_merge_plan: bad sizes");
  if (num_src > kScanBlock * 1024 || num_dst + 1 > kScanBlock * 1024)
    return fail(GPA_ERR_UNSUPPORTED, "gpa_merge_plan: more than 1048576 src or dst tokens");
  if (r > num_src) r = num_src;
  const int unm_len = num_src - r;
  int64_t need = gpa_merge_plan_workspace_bytes(num_src, num_dst);
  if (!workspace || workspace_bytes < need)
    return fail(GPA_ERR_INVALID, "gpa_merge_plan: workspace too small");
  if (!seg_start || !counts || (num_src && (!node_max || !node_idx)) || (r && !seg_src) ||
      (unm_len && !unm_src))
    return fail(GPA_ERR_INVALID, "gpa_merge_plan: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  PlanWs w;
  plan_ws_layout(num_src, num_dst, (char*)workspace, &w);
  const int nb = (num_src + 255) / 256;
  int launched = 0;

  cudaError_t me = cudaSuccess;
  // 1. which src are merged
  if (r == num_src) {
    if (num_src) { fill_ones_kernel<<<nb, 256, 0, st>>>(w.flags, num_src); ++launched; }
  } else if (r == 0) {
    me = cudaMemsetAsync(w.flags, 0, (size_t)num_src * 4, st);
  } else {
    select_init_kernel<<<1, 256, 0, st>>>(w.st, w.hist, (uint32_t)r);
    ++launched;
    int hist_blocks = std::min(1024, (num_src + 1023) / 1024);
    for (int pass = 0; pass < kRadixPasses; ++pass) {
      select_hist_kernel<<<hist_blocks, 256, 0, st>>>(node_max, num_src, pass, w.st, w.hist);
      select_pick_kernel<<<1, 1, 0, st>>>(pass, w.st, w.hist);
      launched += 2;
    }
    select_flags_kernel<<<nb, 256, 0, st>>>(node_max, num_src, w.st, w.flags, w.eq);
    launched += 1 + exclusive_scan<0>(w.eq, w.rank, num_src, w.block_sums, nullptr, st);
    select_final_kernel<<<nb, 256, 0, st>>>(num_src, w.st, w.flags, w.eq, w.rank);
    ++launched;
  }
  // 2. group sizes -> CSR offsets and counts
  if (me == cudaSuccess) me = cudaMemsetAsync(w.seg_len, 0, (size_t)(num_dst + 1) * 4, st);
  if (me != cudaSuccess)
    return fail(GPA_ERR_CUDA, "gpa_merge_plan: cudaMemsetAsync: %s", cudaGetErrorString(me));
  if (num_src) { group_hist_kernel<<<nb, 256, 0, st>>>(node_idx, w.flags, num_src, w.seg_len); ++launched; }
  launched += exclusive_scan<0>(w.seg_len, seg_start, num_dst + 1, w.block_sums, nullptr, st);
  group_counts_kernel<<<(num_dst + 255) / 256, 256, 0, st>>>(seg_start, num_dst, counts, unm_len);
  ++launched;
  // 3. members of each group in ascending src ordinal: compact the merged
  //    (dst, src) pairs in src order, then sort them stably by dst
  if (num_src) {
    int passes = 0;
    for (int bits = 32 - __builtin_clz((unsigned)std::max(num_dst - 1, 1)); bits > 0; bits -= 8) ++passes;
    if (num_dst == 1) passes = 0;   // one group: src order is the answer
    launched += exclusive_scan<0>(w.flags, w.rank, num_src, w.block_sums, nullptr, st);
    int32_t* vals = (passes == 0) ? seg_src : w.val_a;
    group_compact_kernel<<<nb, 256, 0, st>>>(node_idx, w.flags, w.rank, num_src,
                                             passes ? w.key_a : nullptr, vals, unm_src);
    ++launched;
    const int rblk = radix_blocks(r);
    int32_t* kin = w.key_a;
    int32_t* vin = w.val_a;
    int32_t* kalt = (int32_t*)w.eq;
    int32_t* valt = w.val_b;
    for (int pass = 0; pass < passes && r > 0; ++pass) {
      const bool last = pass + 1 == passes;
      int32_t* kout = last ? nullptr : kalt;
      int32_t* vout = last ? seg_src : valt;
      radix_hist_kernel<<<rblk, kRadixDigits, 0, st>>>(kin, r, 8 * pass, rblk, w.table);
      launched += 1 + exclusive_scan<0>(w.table, w.table, kRadixDigits * rblk, w.block_sums, nullptr, st);
      radix_scatter_kernel<<<rblk, 32, 0, st>>>(kin, vin, r, 8 * pass, rblk, w.table, kout, vout);
      ++launched;
      kalt = kin; valt = vin;
      kin = kout; vin = vout;
    }
  }
  if (unm_len) { ones_f32_kernel<<<(unm_len + 255) / 256, 256, 0, st>>>(counts, unm_len); ++launched; }
  return check_launch("gpa_merge_plan", launched);
}

extern "C" int gpa_merge_kv_mean(const void* t, int dtype, int heads, int n_tokens, int head_dim,
                                 int64_t t_stride_h, int64_t t_stride_n, const int32_t* src_pos,
                                 const int32_t* dst_pos, const int32_t* unm_src, int unm_len,
                                 const int32_t* seg_start, const int32_t* seg_src, int num_dst,
                                 int reduce_mean, float* log_counts, void* out,
                                 int64_t out_stride_h, int64_t out_stride_n, void* stream) {
  if (heads <= 0 || head_dim <= 0 || head_dim % 8 || n_tokens <= 0 || unm_len < 0 || num_dst < 0 ||
      unm_len + num_dst <= 0)
    return fail(GPA_ERR_INVALID, "gpa_merge_kv_mean: bad sizes (head_dim %% 8 == 0)");
  if ((unm_len && (!src_pos || !unm_src)) || (num_dst && (!dst_pos || !seg_start || !src_pos)))
    return fail(GPA_ERR_INVALID, "gpa_merge_kv_mean: null index array");
  if (t_stride_h % 8 || t_stride_n % 8 || out_stride_h % 8 || out_stride_n % 8)
    return fail(GPA_ERR_INVALID, "gpa_merge_kv_mean: strides must be multiples of 8 elements");
  if (!aligned16(t) || !aligned16(out))
    return fail(GPA_ERR_INVALID, "gpa_merge_kv_mean: pointers must be 16-byte aligned");
  if (dtype != GPA_DTYPE_F32 && dtype != GPA_DTYPE_BF16)
    return fail(GPA_ERR_INVALID, "gpa_merge_kv_mean: dtype must be f32 or bf16");
  const int nch = heads * head_dim / 8;
  const int slots = unm_len + num_dst;
  cudaStream_t st = (cudaStream_t)stream;
  // staging per warp: two batches of up to kMergeRows rows (2 was fastest in a
  // sweep of 2-4 rows x 2-8 warps per block), at most 8 KB per batch;
  // persistent warps, a few blocks per SM
  const int row_bytes = nch * 8 * (dtype == GPA_DTYPE_BF16 ? 2 : 4);
  const int rows_per_batch = std::max(1, std::min(kMergeRows, 8192 / row_bytes));
  const size_t smem = (size_t)kMergeWarps * 2 * rows_per_batch * row_bytes;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // one wave of resident blocks (persistent warps)
  auto grid_for = [&](const void* fn) {
    int per_sm = 1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kMergeWarps * 32, smem) != cudaSuccess ||
        per_sm < 1)
      per_sm = 1;
    return dim3((unsigned)std::min<int64_t>((slots + kMergeWarps - 1) / kMergeWarps, (int64_t)sms * per_sm));
  };
#define GPA_MERGE_LAUNCH(T, CPL)                                                                  \
  {                                                                                              \
    cudaFuncSetAttribute(merge_mean_kernel<T, CPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                         (int)smem);                                                             \
    const dim3 grid = grid_for((const void*)merge_mean_kernel<T, CPL>);                          \
    merge_mean_kernel<T, CPL><<<grid, kMergeWarps * 32, smem, st>>>(                             \
        (const T*)t, heads, head_dim, t_stride_h, t_stride_n, src_pos, dst_pos, unm_src, unm_len, \
        seg_start, seg_src, num_dst, reduce_mean, log_counts, (T*)out, out_stride_h, out_stride_n, \
        rows_per_batch);                                                                         \
  }
  if (nch <= 32) {
    if (dtype == GPA_DTYPE_BF16) GPA_MERGE_LAUNCH(__nv_bfloat16, 1) else GPA_MERGE_LAUNCH(float, 1)
  } else if (nch <= 128) {
    if (dtype == GPA_DTYPE_BF16) GPA_MERGE_LAUNCH(__nv_bfloat16, 4) else GPA_MERGE_LAUNCH(float, 4)
  } else if (nch <= 256) {
    if (dtype == GPA_DTYPE_BF16) GPA_MERGE_LAUNCH(__nv_bfloat16, 8) else GPA_MERGE_LAUNCH(float, 8)
  } else {
    return fail(GPA_ERR_UNSUPPORTED, "gpa_merge_kv_mean: heads*head_dim > 2048");
  }
#undef GPA_MERGE_LAUNCH
  return check_launch("gpa_merge_kv_mean");
}

// ===========================================================================
// Merge plan without any device allocation.
//
// Some callers of this library cannot allocate device memory when they call
// in: an inference server or plugin host that hands the whole GPU to its own
// memory arena up front (a cudaMalloc there would bypass the arena, can fail
// under memory pressure, and synchronises the device in the middle of
// serving), or an FFI caller that owns no allocator at all.  For them the
// plan's scratch lives in the fixed array below, which the library carries on
// every GPU that loads it, until the process exits.
//
// * Every call looks up the array's device address with cudaGetSymbolAddress
//   on the current device (host code only sees a host-side stand-in under
//   the array's name).  The lookup is host-only and cheap; doing it on every
//   call keeps the address right after a cudaDeviceReset or a new primary
//   context.  The first call on a device may load the library's module onto
//   that device, so make it before any stream capture on that device.
// * Every call on a device shares the one array and leaves its last contents
//   behind; the plan writes or clears every word it reads, so stale contents
//   never leak into a result, but two calls that overlap on the GPU (other
//   streams, other host threads) race on the array.
// * Sizes whose scratch would not fit (gpa_merge_plan_workspace_bytes above
//   GPA_NOALLOC_SCRATCH_BYTES: about 630k src with 210k dst tokens, which
//   covers S=500 frames of 37x37 patches) are rejected with
//   GPA_ERR_UNSUPPORTED before anything is launched.
// ===========================================================================
namespace {
static __device__ __align__(256) unsigned char g_plan_scratch[GPA_NOALLOC_SCRATCH_BYTES];

int plan_scratch_for_current_device(void** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_plan_scratch);
  if (e != cudaSuccess || !p)
    return fail(GPA_ERR_CUDA, "gpa_merge_plan_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
  *out = p;
  return GPA_OK;
}
}  // namespace

extern "C" int gpa_merge_plan_noalloc(const float* node_max, const int32_t* node_idx, int num_src,
                                      int num_dst, int r, int32_t* unm_src, int32_t* seg_start,
                                      int32_t* seg_src, float* counts, void* stream) {
  if (num_src < 0 || num_dst <= 0 || r < 0)
    return fail(GPA_ERR_INVALID, "gpa_merge_plan_noalloc: bad sizes");
  const int64_t need = gpa_merge_plan_workspace_bytes(num_src, num_dst);
  if (need < 0 || need > (int64_t)GPA_NOALLOC_SCRATCH_BYTES)
    return fail(GPA_ERR_UNSUPPORTED,
                "gpa_merge_plan_noalloc: %d src / %d dst tokens need %lld scratch bytes, more than "
                "the library's fixed %lld (use gpa_merge_plan with a workspace)",
                num_src, num_dst, (long long)need, (long long)GPA_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  int rc = plan_scratch_for_current_device(&scratch);
  if (rc) return rc;
  return gpa_merge_plan(node_max, node_idx, num_src, num_dst, r, unm_src, seg_start, seg_src,
                        counts, scratch, (int64_t)GPA_NOALLOC_SCRATCH_BYTES, stream);
}
