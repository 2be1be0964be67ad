// Matching-metric projection, normalisation and src/dst split in one tcgen05
// kernel (replaces merging/merge.py:180-187 and the split of :172-176).
//
//   m    = bf16(x @ proj)        the reference's autocast GEMM rounds its product to bf16
//   row  = bf16(m / ||m||)       fp32 norm and quotient (`norm` runs in fp32 under
//                                autocast), cast to bf16 by the matcher
//   row -> a[src ordinal] or b[dst ordinal], by the role map of gpa_merge_roles
//
// B200 design.  Persistent CTAs walk 128-row tiles of x.  Warp 0 streams
// (x, proj^T) K-chunks of 64 through a 4-stage TMA ring (128B swizzle, no
// multicast); warp 1 issues tcgen05.mma M=128 N=128 K=16 steps into a
// double-buffered fp32 accumulator in TMEM, so one tile's epilogue overlaps
// the next tile's MMAs; warps 2-5 (TMEM lane == row) round, normalise and
// store their rows.  x is read from HBM once (the kernel is HBM-bound: 563 MB
// of x against 72 GFLOP at S=200); proj^T (256 KB) stays hot in L2.
#include "common.cuh"
#include "capi_util.h"

namespace gpa {
namespace proj {

constexpr int BM = 128;
constexpr int BN = 128;                   // the projected width
constexpr int BK = 64;                    // K-chunk (one 128-byte swizzle row)
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;      // 16 KB
constexpr int B_BYTES = BN * BK * 2;      // 16 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_WARPS = 4;
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
constexpr int TMEM_COLS = 2 * BN;

__global__ void __launch_bounds__(THREADS, 1)
    proj_norm_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                     int rows, int kchunks, const int32_t* __restrict__ slot,
                     __nv_bfloat16* __restrict__ a, __nv_bfloat16* __restrict__ b,
                     int* __restrict__ status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* full = bars;                    // [STAGES]
  uint64_t* empty = full + STAGES;          // [STAGES]
  uint64_t* acc_full = empty + STAGES;      // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint64_t* mma_done = acc_empty + 2;       // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int tiles = (rows + BM - 1) / BM;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      bar_init(&full[s], 1);
      bar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      bar_init(&acc_full[i], 1);
      bar_init(&acc_empty[i], EPI_WARPS);
    }
    bar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (elect_one()) {
      tma_prefetch_desc(&map_x);
      tma_prefetch_desc(&map_w);
      int g = 0;
      bool okw = true;
      for (int t = blockIdx.x; okw && t < tiles; t += gridDim.x) {
        for (int kc = 0; kc < kchunks; ++kc, ++g) {
          const int s = g % STAGES;
          if (!wait_bar(&empty[s], ((g / STAGES) & 1) ^ 1, abort_flag, status, kDevTimeout)) {
            okw = false;
            break;
          }
          bar_expect_tx(&full[s], STAGE_BYTES);
          tma_load_2d(&map_x, &full[s], smem + s * STAGE_BYTES, kc * BK, t * BM);
          tma_load_2d(&map_w, &full[s], smem + s * STAGE_BYTES + A_BYTES, kc * BK, 0);
        }
      }
      // every issued copy lands before the CTA may exit
      const unsigned long long t0 = global_ns();
      for (int j = max(0, g - STAGES); j < g; ++j) drain_bar(&full[j % STAGES], (j / STAGES) & 1, t0);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_bf16(BM, BN, false, false);
      int g = 0, i = 0;
      bool okw = true, issued = false;
      for (int t = blockIdx.x; okw && t < tiles; t += gridDim.x, ++i) {
        const int buf = i & 1;
        if (!wait_bar(&acc_empty[buf], ((i >> 1) & 1) ^ 1, abort_flag, status, kDevTimeout)) break;
        const uint32_t d_tmem = tbase + (uint32_t)(buf * BN);
        for (int kc = 0; kc < kchunks; ++kc, ++g) {
          const int s = g % STAGES;
          if (!wait_bar(&full[s], (g / STAGES) & 1, abort_flag, status, kDevTimeout)) {
            okw = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_bf16(d_tmem, sdesc_sw128(a_addr + k * 32, 16, 1024), sdesc_sw128(b_addr + k * 32, 16, 1024),
                      idesc, (kc | k) != 0);
          umma_commit(&empty[s]);
          issued = true;
        }
        if (okw) umma_commit(&acc_full[buf]);
      }
      // every issued MMA completes before the accumulator can be freed
      if (issued) {
        umma_commit(mma_done);
        drain_bar(mma_done, 0, global_ns());
      }
    }
  } else {
    // ---------------- epilogue: round, normalise, split ----------------
    const int quad = warp & 3;              // the TMEM lane quadrant this warp may read
    int i = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      const int buf = i & 1;
      const bool okw = wait_bar(&acc_full[buf], (i >> 1) & 1, abort_flag, status, kDevTimeout);
      if (!__all_sync(0xffffffffu, okw)) break;
      tc_fence_after();
      float v[BN];
      const uint32_t taddr = tbase + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * BN);
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) tmem_ld32f(taddr + c * 32, v + c * 32);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(&acc_empty[buf]);
      const int row = t * BM + quad * 32 + lane;
      if (row >= rows || *abort_flag) continue;
      float ss = 0.f;
#pragma unroll
      for (int c = 0; c < BN; ++c) {
        v[c] = __bfloat162float(__float2bfloat16_rn(v[c]));   // the bf16 product
        ss = fmaf(v[c], v[c], ss);
      }
      const float nrm = __fsqrt_rn(ss);
      const int s = slot[row];
      __nv_bfloat16* dst = s >= 0 ? b + (int64_t)s * BN : a + (int64_t)(-s - 1) * BN;
#pragma unroll
      for (int u = 0; u < BN / 8; ++u) {
        uint4 pk;
        pk.x = pack_bf16x2(__fdiv_rn(v[8 * u + 0], nrm), __fdiv_rn(v[8 * u + 1], nrm));
        pk.y = pack_bf16x2(__fdiv_rn(v[8 * u + 2], nrm), __fdiv_rn(v[8 * u + 3], nrm));
        pk.z = pack_bf16x2(__fdiv_rn(v[8 * u + 4], nrm), __fdiv_rn(v[8 * u + 5], nrm));
        pk.w = pack_bf16x2(__fdiv_rn(v[8 * u + 6], nrm), __fdiv_rn(v[8 * u + 7], nrm));
        reinterpret_cast<uint4*>(dst)[u] = pk;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
}

}  // namespace proj
}  // namespace gpa

extern "C" int gpa_proj_norm_split(const void* x, int64_t x_stride, int rows, int k, const void* proj_t,
                                   const int32_t* slot, void* a, void* b, int* status, void* stream) {
  using namespace gpa;
  using namespace gpa::proj;
  if (rows < 0 || k <= 0 || k % BK || k > 8192)
    return fail(GPA_ERR_INVALID, "gpa_proj_norm_split: need rows >= 0 and k a multiple of 64 up to 8192");
  if (x_stride < k || x_stride % 8)
    return fail(GPA_ERR_INVALID, "gpa_proj_norm_split: x row stride must be >= k and a multiple of 8");
  if (!x || !proj_t || !slot || !aligned16(x) || !aligned16(proj_t) || (a && !aligned16(a)) ||
      (b && !aligned16(b)))
    return fail(GPA_ERR_INVALID, "gpa_proj_norm_split: null or unaligned pointer");
  if (rows == 0) return ok();
  CUtensorMap mx, mw;
  uint64_t dx[2] = {(uint64_t)k, (uint64_t)rows};
  uint64_t sx[2] = {2, (uint64_t)x_stride * 2};
  uint64_t dw[2] = {(uint64_t)k, (uint64_t)BN};
  uint64_t sw[2] = {2, (uint64_t)k * 2};
  uint32_t box[2] = {BK, BM};
  int rc = make_map_bf16(&mx, x, 2, dx, sx, box, CU_TENSOR_MAP_SWIZZLE_128B, "gpa_proj_norm_split(x)");
  if (!rc) rc = make_map_bf16(&mw, proj_t, 2, dw, sw, box, CU_TENSOR_MAP_SWIZZLE_128B, "gpa_proj_norm_split(proj)");
  if (rc) return rc;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaFuncSetAttribute(proj_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
  const int tiles = (rows + BM - 1) / BM;
  proj_norm_kernel<<<std::min(tiles, sms), THREADS, SMEM, (cudaStream_t)stream>>>(
      mx, mw, rows, k / BK, slot, (__nv_bfloat16*)a, (__nv_bfloat16*)b, status);
  return check_launch("gpa_proj_norm_split");
}
