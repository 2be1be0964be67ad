// Early global blocks (frame attention + shared cross-frame K/V set):
// content-adaptive pooling of each frame's patch keys/values, and the exact
// two-partition log-sum-exp combine.
//
// Reference: vggt/layers/attention.py:73-206 (_frame_special_attention), the
// pooling closure _pool at :113-140 and the combine at :164-176.
#include "common.cuh"
#include "capi_util.h"

namespace gpa {
namespace frame {

constexpr int HD = 64;
constexpr int MAX_POOL = 64;
constexpr int MAX_PATCH = 2048;

// One block per (head, frame).  Assignment: argmax over seeds of the cosine
// similarity of the fp32 key (norms clamped at 1e-6); the first seed wins on
// ties (torch.argmax).  Group sums are fp32 in ascending token order, which is
// the order a CPU scatter_add_ uses.
__global__ void __launch_bounds__(256) pool_kernel(const __nv_bfloat16* __restrict__ k,
                                                   const __nv_bfloat16* __restrict__ v, int ph,
                                                   int pw, int ns, int kp, int64_t sh, int64_t sn,
                                                   int num_frames, __nv_bfloat16* __restrict__ pk,
                                                   __nv_bfloat16* __restrict__ pv, int64_t osh,
                                                   int64_t osn, float* __restrict__ pool_size) {
  const int hh = blockIdx.y, s = blockIdx.x;
  const int P = ph * pw + ns;
  const int nh = (ph + kp - 1) / kp, nw = (pw + kp - 1) / kp, npool = nh * nw;
  const int npatch = ph * pw;
  __shared__ float seeds[MAX_POOL][HD + 1];
  __shared__ int assign[MAX_PATCH];
  __shared__ int order[MAX_PATCH];
  __shared__ int gcount[MAX_POOL], gstart[MAX_POOL + 1], gfill[MAX_POOL];
  const __nv_bfloat16* kb = k + (int64_t)hh * sh + ((int64_t)s * P + ns) * sn;
  const __nv_bfloat16* vb = v + (int64_t)hh * sh + ((int64_t)s * P + ns) * sn;

  // normalised seeds: one warp per seed
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int g = warp; g < npool; g += 8) {
    const int iy = g / nw, ix = g - iy * nw;
    const int tok = iy * kp * pw + ix * kp;
    float2 f = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(kb + (int64_t)tok * sn)[lane]);
    float ss = f.x * f.x + f.y * f.y;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float nrm = fmaxf(__fsqrt_rn(ss), 1e-6f);
    seeds[g][2 * lane] = __fdiv_rn(f.x, nrm);
    seeds[g][2 * lane + 1] = __fdiv_rn(f.y, nrm);
  }
  for (int g = threadIdx.x; g < MAX_POOL; g += blockDim.x) { gcount[g] = 0; gfill[g] = 0; }
  __syncthreads();

  // assignment: one thread per patch token
  for (int i = threadIdx.x; i < npatch; i += blockDim.x) {
    float a[HD];
    const uint4* row = reinterpret_cast<const uint4*>(kb + (int64_t)i * sn);
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < HD / 8; ++u) {
      uint4 raw = __ldg(row + u);
      const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float2 f = __bfloat1622float2(e[q]);
        a[8 * u + 2 * q] = f.x;
        a[8 * u + 2 * q + 1] = f.y;
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
    }
    const float nrm = fmaxf(__fsqrt_rn(ss), 1e-6f);
#pragma unroll
    for (int d = 0; d < HD; ++d) a[d] = __fdiv_rn(a[d], nrm);
    float best = -INFINITY;
    int bi = 0;
    for (int g = 0; g < npool; ++g) {
      float dot = 0.f;
#pragma unroll
      for (int d = 0; d < HD; ++d) dot = fmaf(a[d], seeds[g][d], dot);
      if (dot > best) { best = dot; bi = g; }
    }
    assign[i] = bi;
    atomicAdd(&gcount[bi], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int g = 0; g < npool; ++g) { gstart[g] = acc; acc += gcount[g]; }
    gstart[npool] = acc;
  }
  __syncthreads();
  // stable placement by one warp, 32 tokens at a time
  if (warp == 0) {
    for (int c0 = 0; c0 < npatch; c0 += 32) {
      const int i = c0 + lane;
      const int g = i < npatch ? assign[i] : -1 - lane;
      const unsigned same = __match_any_sync(0xffffffffu, g);
      const int rank = __popc(same & ((1u << lane) - 1u));
      if (i < npatch) order[gstart[g] + gfill[g] + rank] = i;
      __syncwarp();
      if (i < npatch && rank == 0) gfill[g] += __popc(same);
      __syncwarp();
    }
  }
  __syncthreads();
  // group means: thread = (group, 8-element chunk), K and V
  for (int w = threadIdx.x; w < npool * (HD / 8); w += blockDim.x) {
    const int g = w >> 3, c = w & 7;
    float ak[8] = {0}, av[8] = {0};
    auto accumulate = [&](const uint4& rk, const uint4& rv) {
      const __nv_bfloat162* ek = reinterpret_cast<const __nv_bfloat162*>(&rk);
      const __nv_bfloat162* ev = reinterpret_cast<const __nv_bfloat162*>(&rv);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float2 fk = __bfloat1622float2(ek[q]), fv = __bfloat1622float2(ev[q]);
        ak[2 * q] += fk.x; ak[2 * q + 1] += fk.y;
        av[2 * q] += fv.x; av[2 * q + 1] += fv.y;
      }
    };
    // member rows four at a time (loads in flight together), summed in order
    const int o0 = gstart[g], o1 = gstart[g + 1];
    int o = o0;
    for (; o + 4 <= o1; o += 4) {
      uint4 rk[4], rv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t tok = order[o + u];
        rk[u] = __ldg(reinterpret_cast<const uint4*>(kb + tok * sn) + c);
        rv[u] = __ldg(reinterpret_cast<const uint4*>(vb + tok * sn) + c);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) accumulate(rk[u], rv[u]);
    }
    for (; o < o1; ++o) {
      const int64_t tok = order[o];
      accumulate(__ldg(reinterpret_cast<const uint4*>(kb + tok * sn) + c),
                 __ldg(reinterpret_cast<const uint4*>(vb + tok * sn) + c));
    }
    const float cnt = (float)gcount[g];
    const float den = fmaxf(cnt, 1.0f);
    uint4 ok4, ov4;
    __nv_bfloat162* ek = reinterpret_cast<__nv_bfloat162*>(&ok4);
    __nv_bfloat162* ev = reinterpret_cast<__nv_bfloat162*>(&ov4);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      ek[q] = __floats2bfloat162_rn(__fdiv_rn(ak[2 * q], den), __fdiv_rn(ak[2 * q + 1], den));
      ev[q] = __floats2bfloat162_rn(__fdiv_rn(av[2 * q], den), __fdiv_rn(av[2 * q + 1], den));
    }
    const int64_t orow = (int64_t)hh * osh + ((int64_t)s * npool + g) * osn;
    reinterpret_cast<uint4*>(pk + orow)[c] = ok4;
    reinterpret_cast<uint4*>(pv + orow)[c] = ov4;
    if (c == 0) pool_size[((int64_t)hh * num_frames + s) * npool + g] = cnt;
  }
}

// o = bf16(bf16(oa*ca) + ob*cb) with ca, cb the normalised partition weights
// rounded to bf16, as the reference's in-place mul_/addcmul_.
__global__ void __launch_bounds__(256) combine_kernel(
    int heads, int frames, int rows, const __nv_bfloat16* __restrict__ oa, int64_t a0, int64_t a1,
    int64_t a2, const float* __restrict__ la, int64_t la0, int64_t la1, int64_t la2,
    const __nv_bfloat16* __restrict__ ob, int64_t b0, int64_t b1, int64_t b2,
    const float* __restrict__ lb, int64_t lb0, int64_t lb1, int64_t lb2, __nv_bfloat16* __restrict__ o,
    int64_t o0, int64_t o1, int64_t o2) {
  // 8 lanes per 64-wide (frame, row, head) row, 8 features (16 bytes) per lane;
  // rows walk (frame, row, head) so token-major tensors stream in memory order
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)heads * frames * rows;
  const int64_t row = gid >> 3;
  if (row >= total) return;
  const int sub = (int)(gid & 7);
  const int hh = (int)(row % heads);
  const int64_t sr = row / heads;
  const int r = (int)(sr % rows);
  const int s = (int)(sr / rows);
  const float xa = __ldg(la + hh * la0 + s * la1 + r * la2);
  const float xb = __ldg(lb + hh * lb0 + s * lb1 + r * lb2);
  const float mx = fmaxf(xa, xb);
  const float wa = exp2f(xa - mx), wb = exp2f(xb - mx);
  const float den = wa + wb;
  // weights rounded to bf16, a*ca rounded to bf16, then + b*cb: the bf16
  // tensor ops of attention.py:164-176
  const float ca = __bfloat162float(__float2bfloat16_rn(wa / den));
  const float cb = __bfloat162float(__float2bfloat16_rn(wb / den));
  const uint4 va = __ldg(reinterpret_cast<const uint4*>(oa + hh * a0 + s * a1 + r * a2 + sub * 8));
  const uint4 vb = __ldg(reinterpret_cast<const uint4*>(ob + hh * b0 + s * b1 + r * b2 + sub * 8));
  const __nv_bfloat162* ea = reinterpret_cast<const __nv_bfloat162*>(&va);
  const __nv_bfloat162* eb = reinterpret_cast<const __nv_bfloat162*>(&vb);
  uint4 vo;
  __nv_bfloat162* eo = reinterpret_cast<__nv_bfloat162*>(&vo);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 fa = __bfloat1622float2(ea[k]), fb = __bfloat1622float2(eb[k]);
    const float t0 = __bfloat162float(__float2bfloat16_rn(fa.x * ca));
    const float t1 = __bfloat162float(__float2bfloat16_rn(fa.y * ca));
    eo[k] = __floats2bfloat162_rn(t0 + fb.x * cb, t1 + fb.y * cb);
  }
  *reinterpret_cast<uint4*>(o + hh * o0 + s * o1 + r * o2 + sub * 8) = vo;
}

}  // namespace frame
}  // namespace gpa

using namespace gpa;

extern "C" int gpa_frame_pool(const void* k, const void* v, int heads, int num_frames, int ph, int pw,
                              int num_special, int kp, int64_t stride_h, int64_t stride_n, void* pk,
                              void* pv, int64_t out_stride_h, int64_t out_stride_n, float* pool_size,
                              void* stream) {
  if (heads <= 0 || num_frames <= 0 || ph <= 0 || pw <= 0 || num_special < 0 || kp <= 0)
    return fail(GPA_ERR_INVALID, "gpa_frame_pool: bad geometry");
  const int nh = (ph + kp - 1) / kp, nw = (pw + kp - 1) / kp;
  if (nh * nw > frame::MAX_POOL || ph * pw > frame::MAX_PATCH)
    return fail(GPA_ERR_UNSUPPORTED, "gpa_frame_pool: at most %d seeds and %d patches per frame",
                frame::MAX_POOL, frame::MAX_PATCH);
  if (stride_n % 8 || stride_h % 8 || out_stride_h % 8 || out_stride_n % 8)
    return fail(GPA_ERR_INVALID, "gpa_frame_pool: strides must be multiples of 8 elements");
  if (!aligned16(k) || !aligned16(v) || !aligned16(pk) || !aligned16(pv) || !pool_size)
    return fail(GPA_ERR_INVALID, "gpa_frame_pool: pointers must be 16-byte aligned");
  dim3 grid(num_frames, heads);
  frame::pool_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, ph, pw, num_special, kp, stride_h, stride_n,
      num_frames, (__nv_bfloat16*)pk, (__nv_bfloat16*)pv, out_stride_h, out_stride_n, pool_size);
  return check_launch("gpa_frame_pool");
}

extern "C" int gpa_lse_combine(int heads, int frames, int rows_per_frame, int head_dim, const void* oa,
                               const int64_t* as, const float* la, const int64_t* las, const void* ob,
                               const int64_t* bs, const float* lb, const int64_t* lbs, void* o,
                               const int64_t* os, void* stream) {
  if (head_dim != 64) return fail(GPA_ERR_UNSUPPORTED, "gpa_lse_combine: head_dim must be 64");
  if (heads <= 0 || frames <= 0 || rows_per_frame <= 0 || !oa || !ob || !o || !la || !lb || !as ||
      !las || !bs || !lbs || !os)
    return fail(GPA_ERR_INVALID, "gpa_lse_combine: bad arguments");
  for (int i = 0; i < 3; ++i)
    if (as[i] % 8 || bs[i] % 8 || os[i] % 8)
      return fail(GPA_ERR_INVALID, "gpa_lse_combine: strides must be multiples of 8 elements");
  if (!aligned16(oa) || !aligned16(ob) || !aligned16(o))
    return fail(GPA_ERR_INVALID, "gpa_lse_combine: 16-byte aligned rows required");
  const int64_t total = (int64_t)heads * frames * rows_per_frame;
  const int64_t blocks = (total * 8 + 255) / 256;   // 8 lanes per row
  if (blocks > 0x7fffffffll) return fail(GPA_ERR_UNSUPPORTED, "gpa_lse_combine: too large");
  frame::combine_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      heads, frames, rows_per_frame, (const __nv_bfloat16*)oa, as[0], as[1], as[2], la, las[0],
      las[1], las[2], (const __nv_bfloat16*)ob, bs[0], bs[1], bs[2], lb, lbs[0], lbs[1], lbs[2],
      (__nv_bfloat16*)o, os[0], os[1], os[2]);
  return check_launch("gpa_lse_combine");
}

// ---------------------------------------------------------------------------
// failure-path self-test: one warp waits on an mbarrier that nothing arrives
// on, through the same bounded wait the pipelined kernels use; the wait gives
// up after limit_ns, records kDevTimeout in *status and the kernel returns.
// Nothing else is in flight, so the context stays usable.
// ---------------------------------------------------------------------------
namespace gpa {
__global__ void wait_selftest_kernel(unsigned long long limit_ns, int* status) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    bar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  wait_bar(&bar, 0, &abort_flag, status, kDevTimeout, limit_ns);
  __syncthreads();
}
}  // namespace gpa

extern "C" int gpa_wait_selftest(uint64_t limit_ns, int* status, void* stream) {
  if (!status) return gpa::fail(GPA_ERR_INVALID, "gpa_wait_selftest: null status word");
  if (limit_ns < 1000 || limit_ns > 10000000000ull)
    return gpa::fail(GPA_ERR_INVALID, "gpa_wait_selftest: limit must be 1 us .. 10 s");
  gpa::wait_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>((unsigned long long)limit_ns, status);
  return gpa::check_launch("gpa_wait_selftest");
}

extern "C" int gpa_version(void) { return 100; }

extern "C" const char* gpa_last_error(void) { return gpa::last_error_buf(); }

extern "C" int64_t gpa_launch_count(void) { return gpa::launch_counter().load(); }
