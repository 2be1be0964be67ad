// Flash attention with a per-key additive bias on the 5th-generation tensor
// cores (head_dim 64, bf16 in, fp32 accumulate).
//
// Reference: merging/fused_attention.py:70-180 (_attn_keybias_kernel and
// attention_keybias): o = softmax(q k^T * scale + bias) v with an online
// softmax in the exp2 domain; optional log2 row sums lse = m + log2(l).
//
// B200 design (one CTA = two 128-query tiles of one (batch, head); 384 threads):
//   warp 0      TMA producer: Q tiles once, then K/V tiles through a 3-stage
//               ring; writes each key tile's bias/scale as a bf16 hi/lo pair
//               (-1e30 past n) for the extra K step of the score MMA.
//   warps 1, 2  MMA issuers, one per query tile t: S_t = Q_t K^T + beta (A
//               and B from shared memory) and O_t += P_t V (P_t from TMEM, V
//               from shared memory); the tensor core takes work from whichever
//               issuer is ready, so one tile's MMAs run while the other tile
//               is in softmax.
//   warps 4-11  two softmax warpgroups, one per query tile, thread == row:
//               S from TMEM -> online softmax -> P (bf16) back into TMEM.
//               The running max only moves when it grows by more than 2^8
//               (lazy rescale of O in TMEM); 2/8 of the exponentials run as a
//               polynomial on the FMA pipe to offload the MUFU unit (16/clk/SM);
//               scale/bias, max and sum use packed fp32x2 and 3-input max with
//               independent accumulators.
//   MMA order:  per tile, S_t(j+1) as soon as softmax t has pulled S_t(j)
//               into registers, O_t += P_t(j) V_j as soon as P_t(j) is in TMEM;
//               the two tiles' issuers are independent warps, so neither
//               waits on the other's progress (a single polling issuer spent
//               most of its time in shared-memory barrier probes, which are
//               slow while the MMAs stream their operands).
//   TMEM (512 columns): S0 0..127, S1 128..255, O0 256..319, O1 320..383,
//                       P0 384..447, P1 448..511 (P: two bf16 per column).
//   The producer/MMA warpgroup gives registers to the softmax warpgroups
//   (setmaxnreg 80 / 208; 96 / 200 in the persistent kernel).
//
// Short key sequences (at most kPersistMaxTiles key tiles, e.g. the 1,374-key
// frame and DINO attention) run attn_persistent_kernel instead: one CTA per SM
// walks (query pair, batch*head) work items with the same roles, pipeline and
// softmax, every barrier phase counted across items and Q double-buffered, so
// one item's epilogue overlaps the next item's Q and K/V loads and first score
// MMAs (200 frames x 16 heads x 1,374 keys: 2.86 -> 2.50 ms).  Long sequences
// keep one CTA per item (the item loop's extra state cost them about 2%).
#include "common.cuh"
#include "capi_util.h"

namespace gpa {
namespace attn {

constexpr int BM = 128;   // queries per tile
constexpr int BN = 128;   // keys per tile
constexpr int HD = 64;    // head dim
// Key tiles by which the producer's bias loads run ahead of their use (a load
// converted right after it was issued stalled the producer on every L2 miss:
// 219,840-key launches ran 15% slower).
#ifndef GPA_ATTN_BIAS_AHEAD
#define GPA_ATTN_BIAS_AHEAD 4
#endif
constexpr int kBiasAhead = GPA_ATTN_BIAS_AHEAD;
static_assert(kBiasAhead >= 1, "bias look-ahead");
#ifndef GPA_ATTN_STAGES
#define GPA_ATTN_STAGES 3
#endif
constexpr int STAGES = GPA_ATTN_STAGES;   // K/V ring depth
constexpr int TILE_BYTES = BM * HD * 2;  // 16 KB
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr int THREADS = 384;
constexpr int TMEM_COLS = 512;
// setmaxnreg split between the producer/MMA warpgroup and the two softmax
// warpgroups: the one-item kernel keeps 80 / 208; the persistent kernel's item
// loop needs 96 in the producer and MMA warps (at 80 they spill), leaving 200.
constexpr int REGS_LAUNCH = 168;
template <bool PERSIST>
struct Regs {
  static constexpr int LOW = PERSIST ? 96 : 80;
  static constexpr int HIGH = (REGS_LAUNCH * 384 - LOW * 128) / 256 / 8 * 8;
  static_assert(LOW * 128 + HIGH * 256 <= REGS_LAUNCH * THREADS, "register split");
};

// Per-key bias as one more K=16 step of S = Q K^T: A_x = [1, 1, 0..] per query
// row, B_x = [hi(beta_j), lo(beta_j), 0..] per key with beta_j = bias_j / scale
// split into two bf16s (about 16 bits), so S' = q.k + beta and
// scale*log2e*S' = q.k*scale*log2e + bias*log2e.  128 x 16 bf16, K-major, no
// swizzle: 8x8 core matrices, rows 16 B apart, K halves LBO=128 B apart, row
// groups SBO=256 B apart.
constexpr int XTILE_BYTES = BM * 16 * 2;  // 4 KB
__host__ __device__ constexpr int xtile_off(int row, int k) {
  return (row >> 3) * 256 + (k >> 3) * 128 + (row & 7) * 16 + (k & 7) * 2;
}
constexpr float kMaskedBeta = -1.0e30f;   // keys past n

// Shared memory: the persistent kernel double-buffers Q (the next item's Q
// lands while this item's last score MMAs read the other buffer).
template <bool PERSIST>
struct SmemT {
  static constexpr int QBUFS = PERSIST ? 2 : 1;
  static constexpr int Q = 0;                               // QBUFS x 2 tiles x 16 KB
  static constexpr int K = Q + QBUFS * 2 * TILE_BYTES;      // STAGES x 16 KB
  static constexpr int V = K + STAGES * TILE_BYTES;         // STAGES x 16 KB
  static constexpr int ONES = V + STAGES * TILE_BYTES;      // 4 KB
  static constexpr int BIAS = ONES + XTILE_BYTES;           // STAGES x 4 KB
  static constexpr int BARS = BIAS + STAGES * XTILE_BYTES;
  static constexpr int TOTAL = BARS + 256;
  static constexpr int ALLOC = TOTAL + 1024;
};
static_assert(SmemT<true>::ALLOC <= 232448, "shared memory per CTA");
static_assert((12 + 2 * STAGES) * 8 + 8 <= 256, "barrier area");

struct Params {
  int m, n, heads;
  int q_pairs, items;   // 256-query pairs per (batch, head); work items = q_pairs * batch * heads
  float scale;        // sm_scale
  float scale_log2;   // sm_scale * log2(e)
  const float* bias;
  int64_t bias_sb, bias_sh;
  __nv_bfloat16* o;
  int64_t o_sb, o_sh, o_sm;
  float* lse;
  int64_t lse_sb, lse_sh;
  // optional second partition of the same softmax, combined in the epilogue
  // (vggt/layers/attention.py:164-176): its normalised output rows and log2
  // row sums; the output may alias comb_o (each row is read before written)
  const __nv_bfloat16* comb_o;
  int64_t comb_sb, comb_sh, comb_sm;
  const float* comb_lse;
  int64_t comb_lse_sb, comb_lse_sh;
  int* status;
};

// How many of each group of 8 exponentials run as the FMA-pipe polynomial
// (the rest on MUFU, 16/clk/SM); 2 was fastest in a sweep of 1-4.
#ifndef GPA_ATTN_POLY_PER8
#define GPA_ATTN_POLY_PER8 2
#endif
constexpr int kPolyPer8 = GPA_ATTN_POLY_PER8;
// Degree of that polynomial: 3 (max relative error 7.7e-5) or 2 (1.7e-3).
#ifndef GPA_ATTN_POLY_DEG
#define GPA_ATTN_POLY_DEG 3
#endif
constexpr int kPolyDeg = GPA_ATTN_POLY_DEG;
// Quarter of a key tile's exponentials after which softmax waits for the
// previous O_t += P_t V (P_t and O_t in TMEM are busy until then).
#ifndef GPA_ATTN_ODONE_Q
#define GPA_ATTN_ODONE_Q 1
#endif
constexpr int kOdoneQuarter = GPA_ATTN_ODONE_Q;
// Key sequences of at most this many 128-key tiles run persistent CTAs.
#ifndef GPA_ATTN_PERSIST_TILES
#define GPA_ATTN_PERSIST_TILES 32
#endif
constexpr int kPersistMaxTiles = GPA_ATTN_PERSIST_TILES;


// no-swizzle K-major descriptor of an extra-step tile
__device__ __forceinline__ uint64_t sdesc_none(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(128 >> 4) << 16;   // LBO: next 8 K-elements
  d |= static_cast<uint64_t>(256 >> 4) << 32;   // SBO: next 8 rows
  d |= static_cast<uint64_t>(1) << 46;          // version; layout type 0 = no swizzle
  return d;
}

// exponentials of one group of 8 shifted scores: the last kPolyPer8 on the FMA pipe
__device__ __forceinline__ void exp8(const float* x, float* e) {
#pragma unroll
  for (int i = 0; i < 8 - kPolyPer8; ++i) e[i] = fast_exp2(x[i]);
#pragma unroll
  for (int i = 8 - kPolyPer8; i + 1 < 8; i += 2) exp2_poly2<kPolyDeg>(x[i], x[i + 1], e[i], e[i + 1]);
  if (kPolyPer8 & 1) e[7] = exp2_poly(x[7]);
}

// The one-item kernel's shared memory and register split.
using Smem = SmemT<false>;
constexpr int REGS_LOW = Regs<false>::LOW, REGS_HIGH = Regs<false>::HIGH;

__global__ void __launch_bounds__(THREADS, 1)
    attn_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                const __grid_constant__ CUtensorMap map_v, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Smem::BARS);
  uint64_t* q_full = bars;                 // 1
  uint64_t* kv_full = bars + 1;            // STAGES
  uint64_t* kv_empty = kv_full + STAGES;   // STAGES
  uint64_t* s_full = kv_empty + STAGES;    // 2
  uint64_t* s_empty = s_full + 2;          // 2
  uint64_t* p_full = s_empty + 2;          // 2
  uint64_t* o_done = p_full + 2;           // 2
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int bh = blockIdx.y;
  const int b = bh / p.heads, h = bh - b * p.heads;
  const int q0 = blockIdx.x * (2 * BM);
  const int nk = (p.n + BN - 1) / BN;

  if (threadIdx.x == 0) {
    bar_init(q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      bar_init(&kv_full[s], 1);
      bar_init(&kv_empty[s], 2);   // one arrival per query tile's issuer
    }
    for (int t = 0; t < 2; ++t) {
      bar_init(&s_full[t], 1);
      bar_init(&s_empty[t], 4);
      bar_init(&p_full[t], 4);
      bar_init(&o_done[t], 1);
    }
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

  if (warp < 4) {
    regs_dec<REGS_LOW>();
    if (warp == 0) {
      // ------------------------------ producer ------------------------------
      const float* brow = p.bias ? p.bias + (int64_t)b * p.bias_sb + (int64_t)h * p.bias_sh : nullptr;
      int issued = 0;
      if (lane == 0) {
        tma_prefetch_desc(&map_q);
        tma_prefetch_desc(&map_k);
        tma_prefetch_desc(&map_v);
        bar_expect_tx(q_full, 2 * TILE_BYTES);
        tma_load_4d(&map_q, q_full, smem + Smem::Q, 0, q0, h, b);
        tma_load_4d(&map_q, q_full, smem + Smem::Q + TILE_BYTES, 0, q0 + BM, h, b);
      }
      // constant A_x tile and zeroed B_x tiles (only columns 0-1 change later)
      {
        uint32_t* w = reinterpret_cast<uint32_t*>(smem + Smem::ONES);
        for (int i = lane; i < (XTILE_BYTES * (1 + STAGES)) / 4; i += 32) w[i] = 0u;
        __syncwarp();
        for (int row = lane; row < BM; row += 32)
          *reinterpret_cast<uint32_t*>(smem + Smem::ONES + xtile_off(row, 0)) = 0x3F803F80u;  // 1, 1
      }
      // The raw bias of key tile j+kBiasAhead is loaded while tile j is staged,
      // so a bias line that misses L2 does not hold up the next TMA issue.
      const float inv_scale = 1.0f / p.scale;
      float braw[kBiasAhead][BN / 32];
      auto load_bias = [&](int j, float* dst) {
#pragma unroll
        for (int i = 0; i < BN / 32; ++i) {
          const int col = j * BN + i * 32 + lane;
          dst[i] = (brow && col < p.n) ? __ldg(brow + col) : 0.0f;
        }
      };
#pragma unroll
      for (int a = 0; a < kBiasAhead; ++a) load_bias(a, braw[a]);
      for (int j = 0; j < nk; ++j) {
        const int s = j % STAGES;
        const uint32_t ph = (j / STAGES) & 1;
        bool okw = wait_bar(&kv_empty[s], ph ^ 1, abort_flag, p.status, kDevTimeout);
        if (!__all_sync(0xffffffffu, okw)) break;
        uint8_t* bt = smem + Smem::BIAS + s * XTILE_BYTES;
#pragma unroll
        for (int i = 0; i < BN / 32; ++i) {
          const int col = j * BN + i * 32 + lane;
          // -inf (or NaN) bias behaves like a key past n
          const float beta = col < p.n ? fmaxf(braw[0][i] * inv_scale, kMaskedBeta) : kMaskedBeta;
          const __nv_bfloat16 hi = __float2bfloat16_rn(beta);
          const __nv_bfloat16 lo = __float2bfloat16_rn(beta - __bfloat162float(hi));
          *reinterpret_cast<uint32_t*>(bt + xtile_off(i * 32 + lane, 0)) =
              (uint32_t)__bfloat16_as_ushort(hi) | ((uint32_t)__bfloat16_as_ushort(lo) << 16);
        }
        fence_async_smem();   // generic-proxy writes -> tensor core reads
        __syncwarp();
        if (lane == 0) {
          bar_expect_tx(&kv_full[s], 2 * TILE_BYTES);
          tma_load_4d(&map_k, &kv_full[s], smem + Smem::K + s * TILE_BYTES, 0, j * BN, h, b);
          tma_load_4d(&map_v, &kv_full[s], smem + Smem::V + s * TILE_BYTES, 0, j * BN, h, b);
        }
        issued = j + 1;
#pragma unroll
        for (int a = 0; a + 1 < kBiasAhead; ++a)
#pragma unroll
          for (int i = 0; i < BN / 32; ++i) braw[a][i] = braw[a + 1][i];
        load_bias(j + kBiasAhead, braw[kBiasAhead - 1]);
      }
      if (lane == 0) {  // drain copies in flight before the CTA can exit
        const unsigned long long t0 = global_ns();
        drain_bar(q_full, 0, t0);
        for (int j = max(0, issued - STAGES); j < issued; ++j)
          drain_bar(&kv_full[j % STAGES], (j / STAGES) & 1, t0);
      }
    } else if (warp == 1 || warp == 2) {
      // ------------------------------ MMA issuers ------------------------------
      // One issuer warp per query tile t (warp 1 -> tile 0, warp 2 -> tile 1),
      // each in order: S_t(j+1) once softmax t holds S_t(j) and K_{j+1} has
      // landed, then O_t += P_t(j) V_j once P_t(j) is in TMEM.  While one
      // issuer waits on its barriers, the other keeps the tensor core fed.
      // Each releases a K/V stage after its PV of that key tile (the empty
      // barrier counts both).  The warp runs the loop converged so descriptor
      // math stays warp-uniform; one elected lane issues and commits.
      // Moving a descriptor by b bytes within shared memory adds b/16 to it.
      const int t = warp - 1;
      const bool leader = elect_one();
      constexpr uint32_t idesc_s = idesc_bf16(BM, BN, false, false);
      constexpr uint32_t idesc_o = idesc_bf16(BM, HD, false, true);
      const uint64_t dQ = sdesc_sw128(smem_u32(smem + Smem::Q + t * TILE_BYTES), 16, 1024);
      const uint64_t dK = sdesc_sw128(smem_u32(smem + Smem::K), 16, 1024);
      const uint64_t dV = sdesc_sw128(smem_u32(smem + Smem::V), 16384, 1024);
      const uint64_t dOnes = sdesc_none(smem_u32(smem + Smem::ONES));
      const uint64_t dBias = sdesc_none(smem_u32(smem + Smem::BIAS));
      const uint32_t dS = tbase + t * BN, dO = tbase + 256 + t * HD, tPm = tbase + 384 + t * 64;
      auto issue_s = [&](int j) {
        const int st = j % STAGES;
        const uint64_t bk = dK + (uint64_t)(st * (TILE_BYTES >> 4));
        const uint64_t bb = dBias + (uint64_t)(st * (XTILE_BYTES >> 4));
        if (leader) {
#pragma unroll
          for (int k = 0; k < HD / 16; ++k) umma_bf16(dS, dQ + 2 * k, bk + 2 * k, idesc_s, k != 0);
          umma_bf16(dS, dOnes, bb, idesc_s, 1);  // + beta_j
          umma_commit(&s_full[t]);
        }
        __syncwarp();
      };
      auto issue_o = [&](int j) {
        const uint64_t bv = dV + (uint64_t)((j % STAGES) * (TILE_BYTES >> 4));
        if (leader) {
#pragma unroll
          for (int ks = 0; ks < BN / 16; ++ks)
            umma_bf16_ts(dO, tPm + ks * 8, bv + (uint64_t)(ks * (2048 >> 4)), idesc_o, (j > 0 || ks > 0));
          umma_commit(&o_done[t]);
          umma_commit(&kv_empty[j % STAGES]);
        }
        __syncwarp();
      };
      bool okw = wait_bar(q_full, 0, abort_flag, p.status, kDevTimeout) &&
                 wait_bar(&kv_full[0], 0, abort_flag, p.status, kDevTimeout);
      okw = __all_sync(0xffffffffu, okw);
      if (okw) {
        tc_fence_after();
        issue_s(0);
      }
      for (int j = 0; okw && j < nk; ++j) {
        if (j + 1 < nk) {
          okw = wait_bar(&s_empty[t], j & 1, abort_flag, p.status, kDevTimeout) &&
                wait_bar(&kv_full[(j + 1) % STAGES], ((j + 1) / STAGES) & 1, abort_flag, p.status,
                         kDevTimeout);
          okw = __all_sync(0xffffffffu, okw);
          if (!okw) break;
          tc_fence_after();
          issue_s(j + 1);
        }
        okw = __all_sync(0xffffffffu, wait_bar(&p_full[t], j & 1, abort_flag, p.status, kDevTimeout));
        if (!okw) break;
        tc_fence_after();
        issue_o(j);
      }
    }
  } else {
    regs_inc<REGS_HIGH>();
    // ------------------------------ softmax ------------------------------
    const int t = (warp - 4) >> 2;       // query tile of this warpgroup
    const int quad = warp & 3;           // TMEM lane quadrant
    const int r = quad * 32 + lane;      // row within the tile
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t tS = tbase + lane_off + t * BN;
    const uint32_t tO = tbase + lane_off + 256 + t * HD;
    const uint32_t tP = tbase + lane_off + 384 + t * 64;
    float m_raw = -INFINITY, l = 0.f;   // running max of S' (raw units), row sum
    const float c2 = p.scale_log2;
    bool okw = true;
    // 32 keys of one row: y = c*(x - m) (packed FMA, in place), P = 2^y (MUFU /
    // polynomial), row-sum accumulators, bf16 pairs
    auto quarter = [&](float* xq, float neg_mc, float* acc, uint32_t* pk) {
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        float* xg = xq + g * 8;
#pragma unroll
        for (int i = 0; i < 8; i += 2) ffma2(xg[i], xg[i + 1], xg[i], xg[i + 1], c2, c2, neg_mc, neg_mc);
        float e[8];
        exp8(xg, e);
#pragma unroll
        for (int i = 0; i < 8; i += 2) fadd2(acc[i], acc[i + 1], acc[i], acc[i + 1], e[i], e[i + 1]);
#pragma unroll
        for (int i = 0; i < 4; ++i) pk[g * 4 + i] = pack_bf16x2(e[2 * i], e[2 * i + 1]);
      }
    };
    auto rescale_o = [&](float alpha) {
      uint32_t ov[32];
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        tmem_ld32(tO + hf * 32, ov);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
        tmem_st32(tO + hf * 32, ov);
      }
    };
    for (int j = 0; j < nk; ++j) {
      okw = wait_bar(&s_full[t], j & 1, abort_flag, p.status, kDevTimeout);
      if (!__all_sync(0xffffffffu, okw)) { okw = false; break; }
      tc_fence_after();
      // x holds S' = q.k + beta (raw units); max on the raw scores
      float x[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) tmem_ld32f(tS + c * 32, x + c * 32);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(&s_empty[t]);
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < BN / 4; ++c) {
        mx[c & 3] = fmax3(mx[c & 3], x[4 * c + 0], x[4 * c + 1]);
        mx[c & 3] = fmax3(mx[c & 3], x[4 * c + 2], x[4 * c + 3]);
      }
      const float mt = fmax3(fmaxf(mx[0], mx[1]), mx[2], mx[3]);
      float alpha = 1.f;
      const bool moved = (mt - m_raw) * c2 > kRescaleThreshold;  // also when m_raw = -inf
      if (moved) {
        alpha = fast_exp2((m_raw - mt) * c2);  // 0 on the first tile
        l *= alpha;
        m_raw = mt;
      }
      const float neg_mc = -m_raw * c2;
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      uint32_t pk[4][16];   // packed bf16 pairs, 32 keys per quarter
#pragma unroll
      for (int qt = 0; qt < 4; ++qt) {
        quarter(x + qt * 32, neg_mc, acc, pk[qt]);
        // P_t and O_t are free once the previous O_t += P_t V finished; the
        // first kOdoneQuarter+1 quarters of the exponentials hide that wait
        if (qt == kOdoneQuarter) {
          if (j > 0) {
            okw = wait_bar(&o_done[t], (j - 1) & 1, abort_flag, p.status, kDevTimeout);
            if (!__all_sync(0xffffffffu, okw)) { okw = false; break; }
            tc_fence_after();
          }
#pragma unroll
          for (int u = 0; u <= kOdoneQuarter; ++u) tmem_st16(tP + u * 16, pk[u]);
        } else if (qt > kOdoneQuarter) {
          tmem_st16(tP + qt * 16, pk[qt]);
        }
      }
      if (!okw) break;
      l += ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
      // rescale O_t in TMEM where the running max moved
      if (j > 0 && __any_sync(0xffffffffu, moved)) rescale_o(alpha);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(&p_full[t]);
    }
    // epilogue
    if (okw) {
      okw = wait_bar(&o_done[t], (nk - 1) & 1, abort_flag, p.status, kDevTimeout);
      okw = __all_sync(0xffffffffu, okw);
    }
    if (okw) {
      tc_fence_after();
      uint32_t ov[HD];
      tmem_ld32(tO, ov);
      tmem_ld32(tO + 32, ov + 32);
      tmem_wait_ld();
      const int row = q0 + t * BM + r;
      if (row < p.m && !*abort_flag) {
        float lse_row = m_raw * p.scale_log2 + __log2f(l);
        float cb = 1.0f / l;   // weight of this partition's unnormalised O
        __nv_bfloat16* orow = p.o + (int64_t)b * p.o_sb + (int64_t)h * p.o_sh + (int64_t)row * p.o_sm;
        if (p.comb_o) {
          // exact two-partition softmax: o = (wa*oa + wb*ob) / (wa + wb) with
          // wa = 2^(lse_a - mx), wb = 2^(lse_b - mx), ob = O / l
          const float la = p.comb_lse[(int64_t)b * p.comb_lse_sb + (int64_t)h * p.comb_lse_sh + row];
          const float mx = fmaxf(la, lse_row);
          const float wa = exp2f(la - mx), wb = exp2f(lse_row - mx);
          const float inv = 1.0f / (wa + wb);
          const float ca = wa * inv;
          cb = wb * inv * cb;
          lse_row = mx + __log2f(wa + wb);
          const uint4* arow = reinterpret_cast<const uint4*>(
              p.comb_o + (int64_t)b * p.comb_sb + (int64_t)h * p.comb_sh + (int64_t)row * p.comb_sm);
          uint4 oa[HD / 8];
#pragma unroll
          for (int u = 0; u < HD / 8; ++u) oa[u] = arow[u];   // the whole row before any store
#pragma unroll
          for (int u = 0; u < HD / 8; ++u) {
            const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&oa[u]);
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float2 f = __bfloat1622float2(e[i]);
              w[i] = pack_bf16x2(fmaf(cb, __uint_as_float(ov[8 * u + 2 * i]), ca * f.x),
                                 fmaf(cb, __uint_as_float(ov[8 * u + 2 * i + 1]), ca * f.y));
            }
            reinterpret_cast<uint4*>(orow)[u] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        } else {
#pragma unroll
          for (int u = 0; u < HD / 8; ++u) {
            uint4 pk;
            pk.x = pack_bf16x2(__uint_as_float(ov[8 * u + 0]) * cb, __uint_as_float(ov[8 * u + 1]) * cb);
            pk.y = pack_bf16x2(__uint_as_float(ov[8 * u + 2]) * cb, __uint_as_float(ov[8 * u + 3]) * cb);
            pk.z = pack_bf16x2(__uint_as_float(ov[8 * u + 4]) * cb, __uint_as_float(ov[8 * u + 5]) * cb);
            pk.w = pack_bf16x2(__uint_as_float(ov[8 * u + 6]) * cb, __uint_as_float(ov[8 * u + 7]) * cb);
            reinterpret_cast<uint4*>(orow)[u] = pk;
          }
        }
        if (p.lse) p.lse[(int64_t)b * p.lse_sb + (int64_t)h * p.lse_sh + row] = lse_row;
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

// Runs body(item) for this CTA's work items: blockIdx.x, + gridDim.x, ...
// while the body returns true (or the one item blockIdx.x).
template <bool PERSIST, typename F>
__device__ __forceinline__ void for_items(int items, F&& body) {
  if constexpr (PERSIST) {
    for (int it = blockIdx.x; it < items; it += gridDim.x)
      if (!body(it)) return;
  } else {
    body((int)blockIdx.x);
  }
}

// The persistent kernel, for short key sequences: one CTA per SM walks work
// items; the same roles, pipeline and softmax as attn_kernel, with every
// barrier phase counted across the CTA's items and Q double-buffered.
__global__ void __launch_bounds__(THREADS, 1)
    attn_persistent_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                           const __grid_constant__ CUtensorMap map_v, const Params p) {
  constexpr bool PERSIST = true;
  using Smem = SmemT<PERSIST>;
  constexpr int REGS_LOW = Regs<PERSIST>::LOW, REGS_HIGH = Regs<PERSIST>::HIGH;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Smem::BARS);
  uint64_t* q_full = bars;                 // 2 (Q buffers)
  uint64_t* q_empty = bars + 2;            // 2
  uint64_t* kv_full = bars + 4;            // STAGES
  uint64_t* kv_empty = kv_full + STAGES;   // STAGES
  uint64_t* s_full = kv_empty + STAGES;    // 2
  uint64_t* s_empty = s_full + 2;          // 2
  uint64_t* p_full = s_empty + 2;          // 2
  uint64_t* o_done = p_full + 2;           // 2
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int nk = (p.n + BN - 1) / BN;
  // Work items: (query pair, batch*head), the query pair fastest, so the CTAs
  // running at one time share a head's K/V in L2.  A CTA walks items
  // blockIdx.x, + gridDim.x, ...; every barrier phase below counts across its
  // items (key tiles J, K/V stages g, Q buffer fills), so the next item's Q,
  // K/V and first score MMA overlap this item's last tiles and epilogue.
  struct Item {
    int b, h, q0;
  };
  auto item_of = [&](int it) {
    Item w;
    const int bh = it / p.q_pairs;
    w.b = bh / p.heads;
    w.h = bh - w.b * p.heads;
    w.q0 = (it - bh * p.q_pairs) * (2 * BM);
    return w;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      bar_init(&q_full[i], 1);
      bar_init(&q_empty[i], 2);    // the last score MMAs of both query tiles
    }
    for (int s = 0; s < STAGES; ++s) {
      bar_init(&kv_full[s], 1);
      bar_init(&kv_empty[s], 2);   // one arrival per query tile's issuer
    }
    for (int t = 0; t < 2; ++t) {
      bar_init(&s_full[t], 1);
      bar_init(&s_empty[t], 4);
      bar_init(&p_full[t], 4);
      bar_init(&o_done[t], 1);
    }
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

  if (warp < 4) {
    regs_dec<REGS_LOW>();
    if (warp == 0) {
      // ------------------------------ producer ------------------------------
      if (lane == 0) {
        tma_prefetch_desc(&map_q);
        tma_prefetch_desc(&map_k);
        tma_prefetch_desc(&map_v);
      }
      // The raw bias of key tile j+kBiasAhead is loaded while tile j is staged,
      // so a bias line that misses L2 does not hold up the next TMA issue.
      const float inv_scale = 1.0f / p.scale;
      float braw[kBiasAhead][BN / 32];
      int g = 0;          // K/V stages issued (all items)
      int q_fills = 0;    // Q buffer fills issued
      bool okp = true;
      for_items<PERSIST>(p.items, [&](int it) -> bool {
        const Item w = item_of(it);
        const float* brow = p.bias ? p.bias + (int64_t)w.b * p.bias_sb + (int64_t)w.h * p.bias_sh : nullptr;
        auto load_bias = [&](int j, float* dst) {
#pragma unroll
          for (int i = 0; i < BN / 32; ++i) {
            const int col = j * BN + i * 32 + lane;
            dst[i] = (brow && col < p.n) ? __ldg(brow + col) : 0.0f;
          }
        };
        // Q buffer q_fills & 1 is free once the score MMAs of the item two back
        // have completed
        const int qb = q_fills & 1, use = q_fills >> 1;
        if (PERSIST && use > 0) {
          okp = __all_sync(0xffffffffu, wait_bar(&q_empty[qb], (use - 1) & 1, abort_flag, p.status, kDevTimeout));
          if (!okp) return false;
        }
        if (lane == 0) {
          uint8_t* qs = smem + Smem::Q + qb * 2 * TILE_BYTES;
          bar_expect_tx(&q_full[qb], 2 * TILE_BYTES);
          tma_load_4d(&map_q, &q_full[qb], qs, 0, w.q0, w.h, w.b);
          tma_load_4d(&map_q, &q_full[qb], qs + TILE_BYTES, 0, w.q0 + BM, w.h, w.b);
        }
        ++q_fills;
        if (q_fills == 1) {
          // constant A_x tile and zeroed B_x tiles (only columns 0-1 change
          // later), written while the first Q tiles are in flight
          uint32_t* z = reinterpret_cast<uint32_t*>(smem + Smem::ONES);
          for (int i = lane; i < (XTILE_BYTES * (1 + STAGES)) / 4; i += 32) z[i] = 0u;
          __syncwarp();
          for (int row = lane; row < BM; row += 32)
            *reinterpret_cast<uint32_t*>(smem + Smem::ONES + xtile_off(row, 0)) = 0x3F803F80u;  // 1, 1
        }
#pragma unroll
        for (int a = 0; a < kBiasAhead; ++a) load_bias(a, braw[a]);
        for (int j = 0; j < nk; ++j) {
          const int s = g % STAGES;
          const uint32_t ph = (g / STAGES) & 1;
          okp = __all_sync(0xffffffffu, wait_bar(&kv_empty[s], ph ^ 1, abort_flag, p.status, kDevTimeout));
          if (!okp) break;
          uint8_t* bt = smem + Smem::BIAS + s * XTILE_BYTES;
#pragma unroll
          for (int i = 0; i < BN / 32; ++i) {
            const int col = j * BN + i * 32 + lane;
            // -inf (or NaN) bias behaves like a key past n
            const float beta = col < p.n ? fmaxf(braw[0][i] * inv_scale, kMaskedBeta) : kMaskedBeta;
            const __nv_bfloat16 hi = __float2bfloat16_rn(beta);
            const __nv_bfloat16 lo = __float2bfloat16_rn(beta - __bfloat162float(hi));
            *reinterpret_cast<uint32_t*>(bt + xtile_off(i * 32 + lane, 0)) =
                (uint32_t)__bfloat16_as_ushort(hi) | ((uint32_t)__bfloat16_as_ushort(lo) << 16);
          }
          fence_async_smem();   // generic-proxy writes -> tensor core reads
          __syncwarp();
          if (lane == 0) {
            bar_expect_tx(&kv_full[s], 2 * TILE_BYTES);
            tma_load_4d(&map_k, &kv_full[s], smem + Smem::K + s * TILE_BYTES, 0, j * BN, w.h, w.b);
            tma_load_4d(&map_v, &kv_full[s], smem + Smem::V + s * TILE_BYTES, 0, j * BN, w.h, w.b);
          }
          ++g;
#pragma unroll
          for (int a = 0; a + 1 < kBiasAhead; ++a)
#pragma unroll
            for (int i = 0; i < BN / 32; ++i) braw[a][i] = braw[a + 1][i];
          load_bias(j + kBiasAhead, braw[kBiasAhead - 1]);
        }
        return okp;
      });
      if (lane == 0) {  // drain copies in flight before the CTA can exit
        const unsigned long long t0 = global_ns();
        for (int k = max(0, q_fills - 2); k < q_fills; ++k) drain_bar(&q_full[k & 1], (k >> 1) & 1, t0);
        for (int k = max(0, g - STAGES); k < g; ++k) drain_bar(&kv_full[k % STAGES], (k / STAGES) & 1, t0);
      }
    } else if (warp == 1 || warp == 2) {
      // ------------------------------ MMA issuers ------------------------------
      // One issuer warp per query tile t (warp 1 -> tile 0, warp 2 -> tile 1),
      // each in order: S_t(j+1) once softmax t holds S_t(j) and K_{j+1} has
      // landed, then O_t += P_t(j) V_j once P_t(j) is in TMEM.  While one
      // issuer waits on its barriers, the other keeps the tensor core fed.
      // Each releases a K/V stage after its PV of that key tile (the empty
      // barrier counts both).  The warp runs the loop converged so descriptor
      // math stays warp-uniform; one elected lane issues and commits.
      // Moving a descriptor by b bytes within shared memory adds b/16 to it.
      const int t = warp - 1;
      const bool leader = elect_one();
      constexpr uint32_t idesc_s = idesc_bf16(BM, BN, false, false);
      constexpr uint32_t idesc_o = idesc_bf16(BM, HD, false, true);
      const uint64_t dQ0 = sdesc_sw128(smem_u32(smem + Smem::Q + t * TILE_BYTES), 16, 1024);
      const uint64_t dK = sdesc_sw128(smem_u32(smem + Smem::K), 16, 1024);
      const uint64_t dV = sdesc_sw128(smem_u32(smem + Smem::V), 16384, 1024);
      const uint64_t dOnes = sdesc_none(smem_u32(smem + Smem::ONES));
      const uint64_t dBias = sdesc_none(smem_u32(smem + Smem::BIAS));
      const uint32_t dS = tbase + t * BN, dO = tbase + 256 + t * HD, tPm = tbase + 384 + t * 64;
      // S_t = Q_t K^T + beta for the K/V stage of global stage count g
      auto issue_s = [&](int g, uint64_t dQ) {
        const int st = g % STAGES;
        const uint64_t bk = dK + (uint64_t)(st * (TILE_BYTES >> 4));
        const uint64_t bb = dBias + (uint64_t)(st * (XTILE_BYTES >> 4));
        if (leader) {
#pragma unroll
          for (int k = 0; k < HD / 16; ++k) umma_bf16(dS, dQ + 2 * k, bk + 2 * k, idesc_s, k != 0);
          umma_bf16(dS, dOnes, bb, idesc_s, 1);  // + beta_j
          umma_commit(&s_full[t]);
        }
        __syncwarp();
      };
      // O_t (+)= P_t V for stage count g, key tile j of the item
      auto issue_o = [&](int g, int j) {
        const uint64_t bv = dV + (uint64_t)((g % STAGES) * (TILE_BYTES >> 4));
        if (leader) {
#pragma unroll
          for (int ks = 0; ks < BN / 16; ++ks)
            umma_bf16_ts(dO, tPm + ks * 8, bv + (uint64_t)(ks * (2048 >> 4)), idesc_o, (j > 0 || ks > 0));
          umma_commit(&o_done[t]);
          umma_commit(&kv_empty[g % STAGES]);
        }
        __syncwarp();
      };
      // the item's Q buffer is free once its last score MMA completes
      auto release_q = [&](int qb) {
        if (leader) umma_commit(&q_empty[qb]);
        __syncwarp();
      };
      bool okw = true;
      int J = 0, g0 = 0, fills = 0;   // key tiles, K/V stages and Q fills before this item
      for_items<PERSIST>(p.items, [&](int) -> bool {
        const int qb = fills & 1;
        const uint64_t dQ = dQ0 + (uint64_t)((qb * 2 * TILE_BYTES) >> 4);
        // the S buffer is free once softmax t holds the previous item's last S
        okw = wait_bar(&q_full[qb], (fills >> 1) & 1, abort_flag, p.status, kDevTimeout) &&
              (J == 0 || wait_bar(&s_empty[t], (J - 1) & 1, abort_flag, p.status, kDevTimeout)) &&
              wait_bar(&kv_full[g0 % STAGES], (g0 / STAGES) & 1, abort_flag, p.status, kDevTimeout);
        okw = __all_sync(0xffffffffu, okw);
        if (!okw) return false;
        tc_fence_after();
        issue_s(g0, dQ);
        if (PERSIST && nk == 1) release_q(qb);
        for (int j = 0; okw && j < nk; ++j) {
          if (j + 1 < nk) {
            okw = wait_bar(&s_empty[t], (J + j) & 1, abort_flag, p.status, kDevTimeout) &&
                  wait_bar(&kv_full[(g0 + j + 1) % STAGES], ((g0 + j + 1) / STAGES) & 1, abort_flag,
                           p.status, kDevTimeout);
            okw = __all_sync(0xffffffffu, okw);
            if (!okw) break;
            tc_fence_after();
            issue_s(g0 + j + 1, dQ);
            if (PERSIST && j + 2 == nk) release_q(qb);
          }
          okw = __all_sync(0xffffffffu, wait_bar(&p_full[t], (J + j) & 1, abort_flag, p.status, kDevTimeout));
          if (!okw) break;
          tc_fence_after();
          issue_o(g0 + j, j);
        }
        J += nk;
        g0 += nk;
        ++fills;
        return okw;
      });
    }
  } else {
    regs_inc<REGS_HIGH>();
    // ------------------------------ softmax ------------------------------
    const int t = (warp - 4) >> 2;       // query tile of this warpgroup
    const int quad = warp & 3;           // TMEM lane quadrant
    const int r = quad * 32 + lane;      // row within the tile
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t tS = tbase + lane_off + t * BN;
    const uint32_t tO = tbase + lane_off + 256 + t * HD;
    const uint32_t tP = tbase + lane_off + 384 + t * 64;
    const float c2 = p.scale_log2;
    bool okw = true;
    // 32 keys of one row: y = c*(x - m) (packed FMA, in place), P = 2^y (MUFU /
    // polynomial), row-sum accumulators, bf16 pairs
    auto quarter = [&](float* xq, float neg_mc, float* acc, uint32_t* pk) {
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        float* xg = xq + g * 8;
#pragma unroll
        for (int i = 0; i < 8; i += 2) ffma2(xg[i], xg[i + 1], xg[i], xg[i + 1], c2, c2, neg_mc, neg_mc);
        float e[8];
        exp8(xg, e);
#pragma unroll
        for (int i = 0; i < 8; i += 2) fadd2(acc[i], acc[i + 1], acc[i], acc[i + 1], e[i], e[i + 1]);
#pragma unroll
        for (int i = 0; i < 4; ++i) pk[g * 4 + i] = pack_bf16x2(e[2 * i], e[2 * i + 1]);
      }
    };
    auto rescale_o = [&](float alpha) {
      uint32_t ov[32];
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        tmem_ld32(tO + hf * 32, ov);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
        tmem_st32(tO + hf * 32, ov);
      }
    };
    int J = 0;   // key tiles of this CTA's earlier items
    for_items<PERSIST>(p.items, [&](int it) -> bool {
    const Item itm = item_of(it);
    const int b = itm.b, h = itm.h, q0 = itm.q0;
    float m_raw = -INFINITY, l = 0.f;   // running max of S' (raw units), row sum
    for (int j = 0; j < nk; ++j) {
      okw = wait_bar(&s_full[t], (J + j) & 1, abort_flag, p.status, kDevTimeout);
      if (!__all_sync(0xffffffffu, okw)) { okw = false; break; }
      tc_fence_after();
      // x holds S' = q.k + beta (raw units); max on the raw scores
      float x[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) tmem_ld32f(tS + c * 32, x + c * 32);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(&s_empty[t]);
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < BN / 4; ++c) {
        mx[c & 3] = fmax3(mx[c & 3], x[4 * c + 0], x[4 * c + 1]);
        mx[c & 3] = fmax3(mx[c & 3], x[4 * c + 2], x[4 * c + 3]);
      }
      const float mt = fmax3(fmaxf(mx[0], mx[1]), mx[2], mx[3]);
      float alpha = 1.f;
      const bool moved = (mt - m_raw) * c2 > kRescaleThreshold;  // also when m_raw = -inf
      if (moved) {
        alpha = fast_exp2((m_raw - mt) * c2);  // 0 on the first tile
        l *= alpha;
        m_raw = mt;
      }
      const float neg_mc = -m_raw * c2;
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      uint32_t pk[4][16];   // packed bf16 pairs, 32 keys per quarter
#pragma unroll
      for (int qt = 0; qt < 4; ++qt) {
        quarter(x + qt * 32, neg_mc, acc, pk[qt]);
        // P_t and O_t are free once the previous O_t += P_t V finished; the
        // first kOdoneQuarter+1 quarters of the exponentials hide that wait
        if (qt == kOdoneQuarter) {
          if (j > 0) {
            okw = wait_bar(&o_done[t], (J + j - 1) & 1, abort_flag, p.status, kDevTimeout);
            if (!__all_sync(0xffffffffu, okw)) { okw = false; break; }
            tc_fence_after();
          }
#pragma unroll
          for (int u = 0; u <= kOdoneQuarter; ++u) tmem_st16(tP + u * 16, pk[u]);
        } else if (qt > kOdoneQuarter) {
          tmem_st16(tP + qt * 16, pk[qt]);
        }
      }
      if (!okw) break;
      l += ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
      // rescale O_t in TMEM where the running max moved
      if (j > 0 && __any_sync(0xffffffffu, moved)) rescale_o(alpha);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(&p_full[t]);
    }
    // epilogue
    if (okw) {
      okw = wait_bar(&o_done[t], (J + nk - 1) & 1, abort_flag, p.status, kDevTimeout);
      okw = __all_sync(0xffffffffu, okw);
    }
    if (okw) {
      tc_fence_after();
      uint32_t ov[HD];
      tmem_ld32(tO, ov);
      tmem_ld32(tO + 32, ov + 32);
      tmem_wait_ld();
      const int row = q0 + t * BM + r;
      if (row < p.m && !*abort_flag) {
        float lse_row = m_raw * p.scale_log2 + __log2f(l);
        float cb = 1.0f / l;   // weight of this partition's unnormalised O
        __nv_bfloat16* orow = p.o + (int64_t)b * p.o_sb + (int64_t)h * p.o_sh + (int64_t)row * p.o_sm;
        if (p.comb_o) {
          // exact two-partition softmax: o = (wa*oa + wb*ob) / (wa + wb) with
          // wa = 2^(lse_a - mx), wb = 2^(lse_b - mx), ob = O / l
          const float la = p.comb_lse[(int64_t)b * p.comb_lse_sb + (int64_t)h * p.comb_lse_sh + row];
          const float mx = fmaxf(la, lse_row);
          const float wa = exp2f(la - mx), wb = exp2f(lse_row - mx);
          const float inv = 1.0f / (wa + wb);
          const float ca = wa * inv;
          cb = wb * inv * cb;
          lse_row = mx + __log2f(wa + wb);
          const uint4* arow = reinterpret_cast<const uint4*>(
              p.comb_o + (int64_t)b * p.comb_sb + (int64_t)h * p.comb_sh + (int64_t)row * p.comb_sm);
          uint4 oa[HD / 8];
#pragma unroll
          for (int u = 0; u < HD / 8; ++u) oa[u] = arow[u];   // the whole row before any store
#pragma unroll
          for (int u = 0; u < HD / 8; ++u) {
            const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&oa[u]);
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float2 f = __bfloat1622float2(e[i]);
              w[i] = pack_bf16x2(fmaf(cb, __uint_as_float(ov[8 * u + 2 * i]), ca * f.x),
                                 fmaf(cb, __uint_as_float(ov[8 * u + 2 * i + 1]), ca * f.y));
            }
            reinterpret_cast<uint4*>(orow)[u] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        } else {
#pragma unroll
          for (int u = 0; u < HD / 8; ++u) {
            uint4 pk;
            pk.x = pack_bf16x2(__uint_as_float(ov[8 * u + 0]) * cb, __uint_as_float(ov[8 * u + 1]) * cb);
            pk.y = pack_bf16x2(__uint_as_float(ov[8 * u + 2]) * cb, __uint_as_float(ov[8 * u + 3]) * cb);
            pk.z = pack_bf16x2(__uint_as_float(ov[8 * u + 4]) * cb, __uint_as_float(ov[8 * u + 5]) * cb);
            pk.w = pack_bf16x2(__uint_as_float(ov[8 * u + 6]) * cb, __uint_as_float(ov[8 * u + 7]) * cb);
            reinterpret_cast<uint4*>(orow)[u] = pk;
          }
        }
        if (p.lse) p.lse[(int64_t)b * p.lse_sb + (int64_t)h * p.lse_sh + row] = lse_row;
      }
    }
    J += nk;
    return okw;
    });
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
}

static int make_map4(CUtensorMap* map, const void* base, int n_rows, int heads, int batch,
                     int64_t s_row, int64_t s_h, int64_t s_b, const char* what) {
  // dims: (head_dim, rows, heads, batch); unused dims get a harmless stride
  uint64_t dims[4] = {(uint64_t)HD, (uint64_t)n_rows, (uint64_t)heads, (uint64_t)batch};
  uint64_t st[4] = {2, (uint64_t)s_row * 2, (uint64_t)s_h * 2, (uint64_t)s_b * 2};
  if (heads == 1) st[2] = (uint64_t)n_rows * s_row * 2;
  if (batch == 1) st[3] = st[2] * (uint64_t)heads;
  if (st[1] == 0 || st[2] == 0 || st[3] == 0)
    return fail(GPA_ERR_UNSUPPORTED, "%s: zero (broadcast) strides are not supported", what);
  uint32_t box[4] = {HD, BM, 1, 1};
  return make_map_bf16(map, base, 4, dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B, what);
}

// The register split needs the kernel to be launched with REGS_LAUNCH
// registers per thread; refuse to launch otherwise (it would never start).
template <bool PERSIST>
static int check_regs() {
  static int checked = 0;
  if (checked) return checked > 0 ? GPA_OK : GPA_ERR_CUDA;
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, PERSIST ? (const void*)attn_persistent_kernel : (const void*)attn_kernel) !=
      cudaSuccess) {
    checked = -1;
    return fail(GPA_ERR_CUDA, "gpa_attention_keybias: cudaFuncGetAttributes failed");
  }
  if (fa.numRegs * THREADS < Regs<PERSIST>::LOW * 128 + Regs<PERSIST>::HIGH * 256) {
    checked = -1;
    return fail(GPA_ERR_CUDA, "gpa_attention_keybias: kernel built with %d registers/thread, "
                "the warpgroup register split needs %d", fa.numRegs, REGS_LAUNCH);
  }
  checked = 1;
  return GPA_OK;
}

}  // namespace attn
}  // namespace gpa

namespace gpa {
namespace attn {
static int launch(const char* what, const void* q, const void* k, const void* v, const float* bias,
                  int batch, int heads, int m, int n, int head_dim, int64_t q_sb, int64_t q_sh,
                  int64_t q_sm, int64_t k_sb, int64_t k_sh, int64_t k_sn, int64_t v_sb, int64_t v_sh,
                  int64_t v_sn, int64_t bias_sb, int64_t bias_sh, float sm_scale, void* o, int64_t o_sb,
                  int64_t o_sh, int64_t o_sm, float* lse, int64_t lse_sb, int64_t lse_sh,
                  const void* comb_o, int64_t comb_sb, int64_t comb_sh, int64_t comb_sm,
                  const float* comb_lse, int64_t comb_lse_sb, int64_t comb_lse_sh, int* status,
                  void* stream) {
  if (head_dim != HD) return fail(GPA_ERR_UNSUPPORTED, "%s: head_dim must be 64", what);
  if (batch <= 0 || heads <= 0 || m < 0 || n <= 0) return fail(GPA_ERR_INVALID, "%s: bad sizes", what);
  if (!q || !k || !v || !o) return fail(GPA_ERR_INVALID, "%s: null pointer", what);
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
    return fail(GPA_ERR_INVALID, "%s: q/k/v/o must be 16-byte aligned", what);
  if (o_sm % 8 || o_sh % 8 || o_sb % 8)
    return fail(GPA_ERR_INVALID, "%s: o strides must be multiples of 8", what);
  if (comb_o && (!comb_lse || !aligned16(comb_o) || comb_sm % 8 || comb_sh % 8 || comb_sb % 8))
    return fail(GPA_ERR_INVALID, "%s: combine rows need their lse, 16-byte alignment and strides "
                "that are multiples of 8", what);
  if (m == 0) return ok();
  if ((int64_t)batch * heads > 65535) return fail(GPA_ERR_UNSUPPORTED, "%s: batch*heads > 65535", what);
  const int64_t q_pairs = (m + 2 * BM - 1) / (2 * BM);
  const int64_t items = q_pairs * batch * heads;
  const bool persist = (n + BN - 1) / BN <= kPersistMaxTiles;
  int rc = persist ? check_regs<true>() : check_regs<false>();
  if (rc) return rc;
  CUtensorMap mq, mk, mv;
  rc = make_map4(&mq, q, m, heads, batch, q_sm, q_sh, q_sb, what);
  if (!rc) rc = make_map4(&mk, k, n, heads, batch, k_sn, k_sh, k_sb, what);
  if (!rc) rc = make_map4(&mv, v, n, heads, batch, v_sn, v_sh, v_sb, what);
  if (rc) return rc;
  Params p;
  p.m = m; p.n = n; p.heads = heads;
  p.q_pairs = (int)q_pairs; p.items = (int)items;
  p.scale = sm_scale;
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.bias = bias; p.bias_sb = bias_sb; p.bias_sh = bias_sh;
  p.o = (__nv_bfloat16*)o; p.o_sb = o_sb; p.o_sh = o_sh; p.o_sm = o_sm;
  p.lse = lse; p.lse_sb = lse_sb; p.lse_sh = lse_sh;
  p.comb_o = (const __nv_bfloat16*)comb_o; p.comb_sb = comb_sb; p.comb_sh = comb_sh; p.comb_sm = comb_sm;
  p.comb_lse = comb_o ? comb_lse : nullptr; p.comb_lse_sb = comb_lse_sb; p.comb_lse_sh = comb_lse_sh;
  p.status = status;

  // Short key sequences run persistent CTAs, one per SM, each walking work
  // items, so set-up, pipeline fill and epilogue overlap the next item; long
  // ones run one CTA per item.
  if (persist) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaFuncSetAttribute(attn_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SmemT<true>::ALLOC);
    attn_persistent_kernel<<<(int)std::min<int64_t>(items, sms), THREADS, SmemT<true>::ALLOC,
                             (cudaStream_t)stream>>>(mq, mk, mv, p);
  } else {
    cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem::ALLOC);
    dim3 grid((unsigned)q_pairs, (unsigned)(batch * heads));
    attn_kernel<<<grid, THREADS, Smem::ALLOC, (cudaStream_t)stream>>>(mq, mk, mv, p);
  }
  return check_launch(what);
}
}  // namespace attn
}  // namespace gpa

extern "C" int gpa_attention_keybias(const void* q, const void* k, const void* v, const float* bias,
                                     int batch, int heads, int m, int n, int head_dim, int64_t q_sb,
                                     int64_t q_sh, int64_t q_sm, int64_t k_sb, int64_t k_sh,
                                     int64_t k_sn, int64_t v_sb, int64_t v_sh, int64_t v_sn,
                                     int64_t bias_sb, int64_t bias_sh, float sm_scale, void* o,
                                     int64_t o_sb, int64_t o_sh, int64_t o_sm, float* lse,
                                     int64_t lse_sb, int64_t lse_sh, int* status, void* stream) {
  return gpa::attn::launch("gpa_attention_keybias", q, k, v, bias, batch, heads, m, n, head_dim, q_sb,
                           q_sh, q_sm, k_sb, k_sh, k_sn, v_sb, v_sh, v_sn, bias_sb, bias_sh, sm_scale, o,
                           o_sb, o_sh, o_sm, lse, lse_sb, lse_sh, nullptr, 0, 0, 0, nullptr, 0, 0,
                           status, stream);
}

extern "C" int gpa_attention_keybias_combine(
    const void* q, const void* k, const void* v, const float* bias, int batch, int heads, int m, int n,
    int head_dim, int64_t q_sb, int64_t q_sh, int64_t q_sm, int64_t k_sb, int64_t k_sh, int64_t k_sn,
    int64_t v_sb, int64_t v_sh, int64_t v_sn, int64_t bias_sb, int64_t bias_sh, float sm_scale,
    const void* oa, int64_t oa_sb, int64_t oa_sh, int64_t oa_sm, const float* lse_a, int64_t lse_a_sb,
    int64_t lse_a_sh, void* o, int64_t o_sb, int64_t o_sh, int64_t o_sm, float* lse, int64_t lse_sb,
    int64_t lse_sh, int* status, void* stream) {
  if (!oa || !lse_a) return gpa::fail(GPA_ERR_INVALID, "gpa_attention_keybias_combine: null partition");
  return gpa::attn::launch("gpa_attention_keybias_combine", q, k, v, bias, batch, heads, m, n,
                           head_dim, q_sb, q_sh, q_sm, k_sb, k_sh, k_sn, v_sb, v_sh, v_sn, bias_sb,
                           bias_sh, sm_scale, o, o_sb, o_sh, o_sm, lse, lse_sb, lse_sh, oa, oa_sb,
                           oa_sh, oa_sm, lse_a, lse_a_sb, lse_a_sh, status, stream);
}
