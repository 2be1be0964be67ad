// Fused similarity + row argmax on the 5th-generation tensor cores.
//
// Reference: merging/fused_similarity.py:33-112 (_sim_argmax_kernel and
// fused_similarity_argmax): node_max[i], node_idx[i] = max / first argmax over
// j of a_i . b_j, bf16 inputs, fp32 accumulation, strict '>' across tiles.
//
// B200 design: one CTA owns NSUB x 128 rows of a (kept in shared memory for
// the whole kernel) and streams 128-row tiles of b through a TMA ring.  One
// thread issues tcgen05.mma (M=128, N=128, K=16 steps) into a double-buffered
// fp32 score tile in TMEM; 4*NSUB epilogue warps read their rows straight out
// of TMEM (TMEM lane == row) and keep a running max / first index in
// registers.  The M x N score matrix never leaves the SM.
#include "common.cuh"
#include "capi_util.h"

namespace gpa {
namespace sim {

constexpr int BM = 128;          // rows per a-subtile (MMA M)
constexpr int BN = 128;          // rows of b per tile (MMA N)
constexpr int CHUNK_BYTES = BM * 64 * 2;  // one 128 x 64 bf16 swizzled chunk (16 KB)

template <int KC>
struct Cfg {
  static constexpr int NSUB = KC <= 2 ? 2 : 1;             // a-subtiles per CTA
  static constexpr int A_BYTES = NSUB * KC * CHUNK_BYTES;
  static constexpr int B_BYTES = KC * CHUNK_BYTES;          // one b stage
  static constexpr int STAGES = (KC == 1) ? 6 : (KC == 2 ? 4 : (KC == 3 ? 2 : 2));
  static constexpr int SMEM = A_BYTES + STAGES * B_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr int EPI_WARPS = 4 * NSUB;
  static constexpr int THREADS = 64 + EPI_WARPS * 32;       // producer, mma, epilogue
  static constexpr int TMEM_COLS = NSUB * 2 * BN;           // double-buffered scores
};

template <int KC>
__global__ void __launch_bounds__(Cfg<KC>::THREADS, 1)
    sim_argmax_kernel(const __grid_constant__ CUtensorMap map_a,
                      const __grid_constant__ CUtensorMap map_b, int m, int n,
                      float* __restrict__ node_max, int32_t* __restrict__ node_idx,
                      int* __restrict__ status) {
  using C = Cfg<KC>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + C::STAGES * C::B_BYTES);
  uint64_t* full = bars;                       // [STAGES]
  uint64_t* empty = bars + C::STAGES;          // [STAGES]
  uint64_t* a_full = bars + 2 * C::STAGES;     // [1]
  uint64_t* acc_full = a_full + 1;             // [2]
  uint64_t* acc_empty = acc_full + 2;          // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int batch = blockIdx.y;
  const int m0 = blockIdx.x * (BM * C::NSUB);
  const int ntiles = (n + BN - 1) / BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      bar_init(&full[s], 1);
      bar_init(&empty[s], 1);
    }
    bar_init(a_full, 1);
    for (int i = 0; i < 2; ++i) {
      bar_init(&acc_full[i], 1);
      bar_init(&acc_empty[i], C::EPI_WARPS);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (elect_one()) {
      tma_prefetch_desc(&map_a);
      tma_prefetch_desc(&map_b);
      bar_expect_tx(a_full, C::A_BYTES);
      for (int sub = 0; sub < C::NSUB; ++sub)
        for (int kc = 0; kc < KC; ++kc)
          tma_load_3d(&map_a, a_full, sA + (sub * KC + kc) * CHUNK_BYTES, kc * 64, m0 + sub * BM,
                      batch);
      int issued = 0;
      for (int j = 0; j < ntiles; ++j) {
        const int s = j % C::STAGES;
        const uint32_t ph = (j / C::STAGES) & 1;
        if (!wait_bar(&empty[s], ph ^ 1, abort_flag, status, kDevTimeout)) break;
        bar_expect_tx(&full[s], C::B_BYTES);
        for (int kc = 0; kc < KC; ++kc)
          tma_load_3d(&map_b, &full[s], sB + s * C::B_BYTES + kc * CHUNK_BYTES, kc * 64, j * BN,
                      batch);
        issued = j + 1;
      }
      // drain: every issued copy lands before the CTA may exit
      const unsigned long long t0 = global_ns();
      drain_bar(a_full, 0, t0);
      for (int j = max(0, issued - C::STAGES); j < issued; ++j)
        drain_bar(&full[j % C::STAGES], (j / C::STAGES) & 1, t0);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_bf16(BM, BN, false, false);
      bool okw = wait_bar(a_full, 0, abort_flag, status, kDevTimeout);
      for (int j = 0; okw && j < ntiles; ++j) {
        const int s = j % C::STAGES;
        const uint32_t ph = (j / C::STAGES) & 1;
        const int buf = j & 1;
        const uint32_t aph = (j >> 1) & 1;
        if (!wait_bar(&full[s], ph, abort_flag, status, kDevTimeout)) break;
        if (!wait_bar(&acc_empty[buf], aph ^ 1, abort_flag, status, kDevTimeout)) break;
        tc_fence_after();
        for (int sub = 0; sub < C::NSUB; ++sub) {
          const uint32_t d_tmem = tbase + (uint32_t)((sub * 2 + buf) * BN);
#pragma unroll
          for (int kc = 0; kc < KC; ++kc) {
            const uint32_t a_addr = smem_u32(sA + (sub * KC + kc) * CHUNK_BYTES);
            const uint32_t b_addr = smem_u32(sB + s * C::B_BYTES + kc * CHUNK_BYTES);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              umma_bf16(d_tmem, sdesc_sw128(a_addr + k * 32, 16, 1024),
                        sdesc_sw128(b_addr + k * 32, 16, 1024), idesc, (kc | k) != 0);
            }
          }
        }
        umma_commit(&empty[s]);
        umma_commit(&acc_full[buf]);
      }
    }
  } else {
    // ---------------- epilogue: running max / argmax per row ----------------
    const int e = warp - 2;
    const int sub = e >> 2;
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = m0 + sub * BM + quad * 32 + lane;
    float best = -INFINITY;
    int bidx = 0;
    for (int j = 0; j < ntiles; ++j) {
      const int buf = j & 1;
      const uint32_t aph = (j >> 1) & 1;
      const bool okw = wait_bar(&acc_full[buf], aph, abort_flag, status, kDevTimeout);
      if (!__all_sync(0xffffffffu, okw)) break;
      tc_fence_after();
      uint32_t r[BN];
      const uint32_t taddr = tbase + ((uint32_t)(quad * 32) << 16) + (uint32_t)((sub * 2 + buf) * BN);
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) tmem_ld32(taddr + c * 32, r + c * 32);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(&acc_empty[buf]);
      const int col0 = j * BN;
      const int valid = min(BN, n - col0);
      if (valid < BN) {  // last tile: mask the columns past n
#pragma unroll
        for (int i = 0; i < BN; ++i)
          if (i >= valid) r[i] = __float_as_uint(-INFINITY);
      }
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        const uint32_t* rc = r + c * 32;
        // tree of 3-input maxima (short dependency chains)
        float m1[11];
#pragma unroll
        for (int i = 0; i < 10; ++i)
          m1[i] = fmax3(__uint_as_float(rc[3 * i]), __uint_as_float(rc[3 * i + 1]),
                        __uint_as_float(rc[3 * i + 2]));
        m1[10] = fmaxf(__uint_as_float(rc[30]), __uint_as_float(rc[31]));
        const float m2a = fmax3(m1[0], m1[1], m1[2]), m2b = fmax3(m1[3], m1[4], m1[5]);
        const float m2c = fmax3(m1[6], m1[7], m1[8]), m2d = fmaxf(m1[9], m1[10]);
        const float cmax = fmaxf(fmaxf(m2a, m2b), fmaxf(m2c, m2d));
        if (cmax > best) {  // strict: an equal later score keeps the earlier index
          int first = 0;
#pragma unroll
          for (int i = 31; i >= 0; --i)
            if (__uint_as_float(rc[i]) == cmax) first = i;
          best = cmax;
          bidx = col0 + c * 32 + first;
        }
      }
    }
    if (row < m && !*abort_flag) {
      const int64_t o = (int64_t)batch * m + row;
      node_max[o] = best;
      node_idx[o] = bidx;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, C::TMEM_COLS);
  }
}

template <int KC>
static int launch(const void* a, const void* b, int batch, int m, int n, int64_t a_sb,
                  int64_t a_sm, int64_t b_sb, int64_t b_sn, float* node_max, int32_t* node_idx,
                  int* status, cudaStream_t st) {
  using C = Cfg<KC>;
  const int d = KC * 64;
  CUtensorMap ma, mb;
  uint64_t da[3] = {(uint64_t)d, (uint64_t)m, (uint64_t)batch};
  uint64_t sa[3] = {2, (uint64_t)a_sm * 2, (uint64_t)a_sb * 2};
  uint64_t db[3] = {(uint64_t)d, (uint64_t)n, (uint64_t)batch};
  uint64_t sbb[3] = {2, (uint64_t)b_sn * 2, (uint64_t)b_sb * 2};
  uint32_t box[3] = {64, 128, 1};
  if (batch == 1) { sa[2] = (uint64_t)m * a_sm * 2; sbb[2] = (uint64_t)n * b_sn * 2; }
  int rc = make_map_bf16(&ma, a, 3, da, sa, box, CU_TENSOR_MAP_SWIZZLE_128B, "gpa_sim_argmax(a)");
  if (rc) return rc;
  rc = make_map_bf16(&mb, b, 3, db, sbb, box, CU_TENSOR_MAP_SWIZZLE_128B, "gpa_sim_argmax(b)");
  if (rc) return rc;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(sim_argmax_kernel<KC>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    attr_set = true;
  }
  dim3 grid((m + BM * C::NSUB - 1) / (BM * C::NSUB), batch);
  sim_argmax_kernel<KC><<<grid, C::THREADS, C::SMEM, st>>>(ma, mb, m, n, node_max, node_idx, status);
  return check_launch("gpa_sim_argmax");
}

}  // namespace sim
}  // namespace gpa

extern "C" int gpa_sim_argmax(const void* a, const void* b, int batch, int m, int n, int d,
                              int64_t a_stride_b, int64_t a_stride_m, int64_t b_stride_b,
                              int64_t b_stride_n, float* node_max, int32_t* node_idx, int* status,
                              void* stream) {
  using namespace gpa;
  if (batch <= 0 || m < 0 || n <= 0)
    return fail(GPA_ERR_INVALID, "gpa_sim_argmax: need batch > 0, m >= 0, n > 0");
  if (d % 64 || d < 64 || d > 256)
    return fail(GPA_ERR_UNSUPPORTED, "gpa_sim_argmax: d must be 64, 128, 192 or 256 (got %d)", d);
  if (a_stride_m % 8 || b_stride_n % 8 || a_stride_b % 8 || b_stride_b % 8)
    return fail(GPA_ERR_INVALID, "gpa_sim_argmax: strides must be multiples of 8 elements");
  if (!aligned16(a) || !aligned16(b))
    return fail(GPA_ERR_INVALID, "gpa_sim_argmax: a and b must be 16-byte aligned");
  if (!node_max || !node_idx) return fail(GPA_ERR_INVALID, "gpa_sim_argmax: null output");
  if (m == 0) return ok();
  cudaStream_t st = (cudaStream_t)stream;
  switch (d / 64) {
    case 1: return sim::launch<1>(a, b, batch, m, n, a_stride_b, a_stride_m, b_stride_b, b_stride_n, node_max, node_idx, status, st);
    case 2: return sim::launch<2>(a, b, batch, m, n, a_stride_b, a_stride_m, b_stride_b, b_stride_n, node_max, node_idx, status, st);
    case 3: return sim::launch<3>(a, b, batch, m, n, a_stride_b, a_stride_m, b_stride_b, b_stride_n, node_max, node_idx, status, st);
    default: return sim::launch<4>(a, b, batch, m, n, a_stride_b, a_stride_m, b_stride_b, b_stride_n, node_max, node_idx, status, st);
  }
}
