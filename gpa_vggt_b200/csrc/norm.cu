// Normalisation work of the attention blocks, fused and HBM-bound:
//  * gpa_layernorm_bf16: LayerNorm of bf16 rows with fp32 statistics and a
//    bf16 result (the value a bf16-autocast Linear receives after the
//    reference's fp32 LayerNorm, vggt/layers/block.py:85-92).
//  * gpa_qk_norm_rope: per-head LayerNorm of q and k (qk_norm) followed by the
//    2D rotary embedding (vggt/layers/attention.py:216-220, rope.py:139-209),
//    in fp32 registers, written back as bf16 -- one pass over the qkv buffer
//    instead of the norm, rotate, concatenate and cast kernels.
//  * gpa_residual_scale_bf16: the residual add of a LayerScale branch,
//    x + y * gamma, in one pass (vggt/layers/block.py:88,94).
//  * gpa_gelu_bf16: the MLP's exact GELU on bf16 activations.
#include "common.cuh"
#include "capi_util.h"

namespace gpa {
namespace norm {


// 8 consecutive parameters (weight or bias) as floats, one or two vector loads.
__device__ __forceinline__ void ldw8(const __nv_bfloat16* p, int i, float* v) {
  const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p + i));
  const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 f = __bfloat1622float2(e[k]);
    v[2 * k] = f.x;
    v[2 * k + 1] = f.y;
  }
}
__device__ __forceinline__ void ldw8(const float* p, int i, float* v) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p + i));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p + i) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// One warp per row; cols % 256 == 0, cols <= 4096 (16-byte vectors per lane).
template <int VPL, typename W>
__global__ void __launch_bounds__(256) layernorm_kernel(const __nv_bfloat16* __restrict__ x,
                                                        int64_t xs, int rows, const W* __restrict__ w,
                                                        const W* __restrict__ b, float eps,
                                                        __nv_bfloat16* __restrict__ out, int64_t os) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  constexpr int C = VPL * 256;
  const __nv_bfloat16* xr = x + (int64_t)row * xs;
  float v[VPL][8];
  float s = 0.f;
#pragma unroll
  for (int u = 0; u < VPL; ++u) {
    uint4 raw = __ldg(reinterpret_cast<const uint4*>(xr) + u * 32 + lane);
    const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(e[i]);
      v[u][2 * i] = f.x;
      v[u][2 * i + 1] = f.y;
      s += f.x + f.y;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / C;
  float q = 0.f;
#pragma unroll
  for (int u = 0; u < VPL; ++u)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float d = v[u][i] - mean;
      q = fmaf(d, d, q);
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float rstd = rsqrtf(q / C + eps);
  __nv_bfloat16* orow = out + (int64_t)row * os;
#pragma unroll
  for (int u = 0; u < VPL; ++u) {
    const int c0 = (u * 32 + lane) * 8;
    float wv[8], bv[8];
    ldw8(w, c0, wv);
    ldw8(b, c0, bv);
    uint4 raw;
    __nv_bfloat162* e = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float y0 = fmaf((v[u][2 * i] - mean) * rstd, wv[2 * i], bv[2 * i]);
      const float y1 = fmaf((v[u][2 * i + 1] - mean) * rstd, wv[2 * i + 1], bv[2 * i + 1]);
      e[i] = __floats2bfloat162_rn(y0, y1);
    }
    reinterpret_cast<uint4*>(orow)[u * 32 + lane] = raw;
  }
}

// Per 64-wide head row of q or k.  Rotary layout: dims 0..31 turn
// with the row coordinate, 32..63 with the column coordinate; inside each half
// the rotate-half pairing (i, i+16).  cos/sin tables: [n_pos, 32] fp32.
template <typename W>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(
    const __nv_bfloat16* __restrict__ qkv, int64_t tok_stride, int64_t q_off, int64_t k_off,
    int tokens, int heads, const W* __restrict__ qw, const W* __restrict__ qb,
    const W* __restrict__ kw, const W* __restrict__ kb, float eps, const int64_t* __restrict__ pos,
    const float* __restrict__ cos_tab, const float* __restrict__ sin_tab, int n_pos,
    __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_out, int64_t out_tok_stride) {
  // 8 lanes per token, 8 consecutive features of every head per lane: the
  // rotary table entries and the norm weights are loaded once per token, and
  // each step keeps the q and k rows of kHeadsPerStep heads in flight (16-byte
  // coalesced loads and stores).  Mean and variance by xor-shuffles inside the
  // 8-lane group; the rotate-half partner (feature i +- 16) is in lane ^ 2.
  constexpr int kHeadsPerStep = 4;   // 2: 0.63 ms, 4: 0.55 ms, 8: 0.79 ms at S=200
  const uint32_t tok = (blockIdx.x * blockDim.x + threadIdx.x) >> 3;   // the launcher bounds tokens * 8
  if (tok >= (uint32_t)tokens) return;   // whole 8-lane groups leave together
  const int lane = threadIdx.x & 31, sub = lane & 7;
  const unsigned gmask = 0xffu << (lane & 24);
  const int64_t tok64 = tok;
  float c[8], sn[8];
  const bool lower = (sub & 3) < 2;     // features 0..15 of a half pair with +16, 16..31 with -16
  if (pos) {
    const int half = sub >> 2, within = (sub & 3) * 8;   // feature offset inside the half
    int p = (int)pos[tok64 * 2 + half];
    p = min(max(p, 0), n_pos - 1);
    const float4* c4 = reinterpret_cast<const float4*>(cos_tab + (int64_t)p * 32 + within);
    const float4* s4 = reinterpret_cast<const float4*>(sin_tab + (int64_t)p * 32 + within);
    const float4 ca = __ldg(c4), cb = __ldg(c4 + 1), sa = __ldg(s4), sb = __ldg(s4 + 1);
    c[0] = ca.x; c[1] = ca.y; c[2] = ca.z; c[3] = ca.w; c[4] = cb.x; c[5] = cb.y; c[6] = cb.z; c[7] = cb.w;
    sn[0] = sa.x; sn[1] = sa.y; sn[2] = sa.z; sn[3] = sa.w; sn[4] = sb.x; sn[5] = sb.y; sn[6] = sb.z; sn[7] = sb.w;
  }
  float qw8[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f}, qb8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float kw8[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f}, kb8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (qw) ldw8(qw, sub * 8, qw8);
  if (qb) ldw8(qb, sub * 8, qb8);
  if (kw) ldw8(kw, sub * 8, kw8);
  if (kb) ldw8(kb, sub * 8, kb8);
  auto one = [&](const uint4 in, const float* wv, const float* bv, __nv_bfloat16* dst) {
    float v[8];
    {
      const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&in);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(e[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    }
    float s = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
    s += __shfl_xor_sync(gmask, s, 1);
    s += __shfl_xor_sync(gmask, s, 2);
    s += __shfl_xor_sync(gmask, s, 4);
    const float mean = s * (1.f / 64.f);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float d = v[i] - mean;
      q = fmaf(d, d, q);
    }
    q += __shfl_xor_sync(gmask, q, 1);
    q += __shfl_xor_sync(gmask, q, 2);
    q += __shfl_xor_sync(gmask, q, 4);
    const float rstd = rsqrtf(q * (1.f / 64.f) + eps);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = fmaf((v[i] - mean) * rstd, wv[i], bv[i]);
    if (pos) {
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float partner = __shfl_xor_sync(gmask, v[i], 2);
        // separate roundings of the two products and the sum, as t*cos + rot(t)*sin
        o[i] = __fadd_rn(__fmul_rn(v[i], c[i]), __fmul_rn(lower ? -partner : partner, sn[i]));
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = o[i];
    }
    uint4 raw;
    __nv_bfloat162* e = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) e[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(dst) = raw;
  };
  const __nv_bfloat16* src = qkv + tok64 * tok_stride + sub * 8;
  const int64_t out_off = tok64 * out_tok_stride + sub * 8;
  for (int h0 = 0; h0 < heads; h0 += kHeadsPerStep) {
    // a step's rows are all loaded before any is stored: the output may alias
    // the input (in place), so later loads could not be hoisted above a store
    uint4 rq[kHeadsPerStep], rk[kHeadsPerStep];
#pragma unroll
    for (int u = 0; u < kHeadsPerStep; ++u)
      if (h0 + u < heads) {
        rq[u] = *reinterpret_cast<const uint4*>(src + q_off + (h0 + u) * 64);
        rk[u] = *reinterpret_cast<const uint4*>(src + k_off + (h0 + u) * 64);
      }
#pragma unroll
    for (int u = 0; u < kHeadsPerStep; ++u)
      if (h0 + u < heads) {
        one(rq[u], qw8, qb8, q_out + out_off + (h0 + u) * 64);
        one(rk[u], kw8, kb8, k_out + out_off + (h0 + u) * 64);
      }
  }
}

}  // namespace norm
}  // namespace gpa

namespace gpa {
namespace norm {

// Residual + LayerScale: out = bf16(x + bf16(y * gamma[c])), the two roundings
// of torch's bf16 `x + y * gamma` (vggt/layers/block.py:88,94 with
// layers/layer_scale.py:21), one pass over x and y instead of a broadcast
// multiply followed by an add.  One thread per 8 bf16 (16-byte vectors).
__global__ void __launch_bounds__(256) residual_scale_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t x_stride, const __nv_bfloat16* __restrict__ y,
    int64_t y_stride, const __nv_bfloat16* __restrict__ gamma, uint32_t vec_per_row, uint32_t total,
    __nv_bfloat16* __restrict__ out, int64_t out_stride) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint32_t r = i / vec_per_row, c = (i - r * vec_per_row) * 8;
    const uint4 xv = *reinterpret_cast<const uint4*>(x + (int64_t)r * x_stride + c);
    const uint4 yv = *reinterpret_cast<const uint4*>(y + (int64_t)r * y_stride + c);
    const uint4 gv = __ldg(reinterpret_cast<const uint4*>(gamma + c));
    const __nv_bfloat162* xa = reinterpret_cast<const __nv_bfloat162*>(&xv);
    const __nv_bfloat162* ya = reinterpret_cast<const __nv_bfloat162*>(&yv);
    const __nv_bfloat162* ga = reinterpret_cast<const __nv_bfloat162*>(&gv);
    uint4 ov;
    __nv_bfloat162* oa = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 xf = __bfloat1622float2(xa[k]), yf = __bfloat1622float2(ya[k]), gf = __bfloat1622float2(ga[k]);
      const __nv_bfloat162 t = __floats2bfloat162_rn(__fmul_rn(yf.x, gf.x), __fmul_rn(yf.y, gf.y));
      const float2 tf = __bfloat1622float2(t);
      oa[k] = __floats2bfloat162_rn(__fadd_rn(xf.x, tf.x), __fadd_rn(xf.y, tf.y));
    }
    *reinterpret_cast<uint4*>(out + (int64_t)r * out_stride + c) = ov;
  }
}

// Exact (erf) GELU of bf16 values, computed as torch does for bf16 tensors:
// fp32 0.5 * x * (1 + erf(x / sqrt(2))) rounded to bf16 (vggt/layers/mlp.py
// with nn.GELU()).  16-byte vectors, grid-stride.
__global__ void __launch_bounds__(256) gelu_kernel(const __nv_bfloat16* __restrict__ x,
                                                   __nv_bfloat16* __restrict__ out, int64_t nvec) {
  const float kInvSqrt2 = 0.70710678118654752440f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(x) + i);
    const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&raw);
    uint4 o;
    __nv_bfloat162* oe = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __bfloat1622float2(e[k]);
      const float g0 = 0.5f * f.x * (1.0f + erff(f.x * kInvSqrt2));
      const float g1 = 0.5f * f.y * (1.0f + erff(f.y * kInvSqrt2));
      oe[k] = __floats2bfloat162_rn(g0, g1);
    }
    reinterpret_cast<uint4*>(out)[i] = o;
  }
}

}  // namespace norm
}  // namespace gpa

using namespace gpa;

extern "C" int gpa_layernorm_bf16(const void* x, int64_t x_stride, int rows, int cols,
                                  const void* weight, const void* bias, int param_dtype, float eps,
                                  void* out, int64_t out_stride, void* stream) {
  if (rows < 0 || cols <= 0 || cols % 256 || cols > 4096)
    return fail(GPA_ERR_UNSUPPORTED, "gpa_layernorm_bf16: cols must be a multiple of 256, <= 4096");
  if (x_stride % 8 || out_stride % 8 || !aligned16(x) || !aligned16(out) || !weight || !bias ||
      !aligned16(weight) || !aligned16(bias))
    return fail(GPA_ERR_INVALID, "gpa_layernorm_bf16: 16-byte aligned rows and weight/bias required");
  if (param_dtype != GPA_DTYPE_F32 && param_dtype != GPA_DTYPE_BF16)
    return fail(GPA_ERR_INVALID, "gpa_layernorm_bf16: weight dtype must be f32 or bf16");
  if (rows == 0) return ok();
  dim3 grid((rows + 7) / 8);
  cudaStream_t st = (cudaStream_t)stream;
  const int vpl = cols / 256;
#define GPA_LN(V, W)                                                                        \
  norm::layernorm_kernel<V, W><<<grid, 256, 0, st>>>((const __nv_bfloat16*)x, x_stride, rows, \
                                                     (const W*)weight, (const W*)bias, eps,    \
                                                     (__nv_bfloat16*)out, out_stride)
#define GPA_LN_V(W)                                                            \
  switch (vpl) {                                                               \
    case 1: GPA_LN(1, W); break;                                               \
    case 2: GPA_LN(2, W); break;                                               \
    case 4: GPA_LN(4, W); break;                                               \
    case 8: GPA_LN(8, W); break;                                               \
    case 16: GPA_LN(16, W); break;                                             \
    default: return fail(GPA_ERR_UNSUPPORTED, "gpa_layernorm_bf16: cols %d", cols); \
  }
  if (param_dtype == GPA_DTYPE_BF16) {
    GPA_LN_V(__nv_bfloat16)
  } else {
    GPA_LN_V(float)
  }
#undef GPA_LN_V
#undef GPA_LN
  return check_launch("gpa_layernorm_bf16");
}

extern "C" int gpa_qk_norm_rope(const void* qkv, int64_t token_stride, int64_t q_offset,
                                int64_t k_offset, int tokens, int heads, int head_dim,
                                const void* q_weight, const void* q_bias, const void* k_weight,
                                const void* k_bias, int param_dtype, float eps,
                                const int64_t* positions, const float* cos_table,
                                const float* sin_table, int n_pos, void* q_out, void* k_out,
                                int64_t out_token_stride, void* stream) {
  if (head_dim != 64) return fail(GPA_ERR_UNSUPPORTED, "gpa_qk_norm_rope: head_dim must be 64");
  if (tokens < 0 || heads <= 0) return fail(GPA_ERR_INVALID, "gpa_qk_norm_rope: bad sizes");
  if (token_stride % 8 || q_offset % 8 || k_offset % 8 || out_token_stride % 8 || !aligned16(qkv) ||
      !aligned16(q_out) || !aligned16(k_out))
    return fail(GPA_ERR_INVALID, "gpa_qk_norm_rope: 16-byte aligned rows required");
  if (positions && (!cos_table || !sin_table || n_pos <= 0))
    return fail(GPA_ERR_INVALID, "gpa_qk_norm_rope: rotary tables missing");
  if (positions && (!aligned16(cos_table) || !aligned16(sin_table)))
    return fail(GPA_ERR_INVALID, "gpa_qk_norm_rope: rotary tables must be 16-byte aligned");
  if ((q_weight && !aligned16(q_weight)) || (q_bias && !aligned16(q_bias)) ||
      (k_weight && !aligned16(k_weight)) || (k_bias && !aligned16(k_bias)))
    return fail(GPA_ERR_INVALID, "gpa_qk_norm_rope: norm weights must be 16-byte aligned");
  if (param_dtype != GPA_DTYPE_F32 && param_dtype != GPA_DTYPE_BF16)
    return fail(GPA_ERR_INVALID, "gpa_qk_norm_rope: weight dtype must be f32 or bf16");
  if ((int64_t)tokens * heads == 0) return ok();
  if ((int64_t)tokens * 8 >= (1ll << 32)) return fail(GPA_ERR_UNSUPPORTED, "gpa_qk_norm_rope: too many tokens");
  const unsigned blocks = (unsigned)(((int64_t)tokens * 8 + 255) / 256);   // 8 lanes per token
  cudaStream_t st = (cudaStream_t)stream;
  if (param_dtype == GPA_DTYPE_BF16)
    norm::qk_norm_rope_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
        (const __nv_bfloat16*)qkv, token_stride, q_offset, k_offset, tokens, heads,
        (const __nv_bfloat16*)q_weight, (const __nv_bfloat16*)q_bias, (const __nv_bfloat16*)k_weight,
        (const __nv_bfloat16*)k_bias, eps, positions, cos_table, sin_table, n_pos,
        (__nv_bfloat16*)q_out, (__nv_bfloat16*)k_out, out_token_stride);
  else
    norm::qk_norm_rope_kernel<float><<<blocks, 256, 0, st>>>(
        (const __nv_bfloat16*)qkv, token_stride, q_offset, k_offset, tokens, heads,
        (const float*)q_weight, (const float*)q_bias, (const float*)k_weight, (const float*)k_bias,
        eps, positions, cos_table, sin_table, n_pos, (__nv_bfloat16*)q_out, (__nv_bfloat16*)k_out,
        out_token_stride);
  return check_launch("gpa_qk_norm_rope");
}

extern "C" int gpa_residual_scale_bf16(const void* x, int64_t x_stride, const void* y, int64_t y_stride,
                                       const void* gamma, int rows, int cols, void* out,
                                       int64_t out_stride, void* stream) {
  if (rows < 0 || cols <= 0 || cols % 8)
    return fail(GPA_ERR_UNSUPPORTED, "gpa_residual_scale_bf16: cols must be a positive multiple of 8");
  if (x_stride % 8 || y_stride % 8 || out_stride % 8 || !aligned16(x) || !aligned16(y) ||
      !aligned16(out) || !aligned16(gamma))
    return fail(GPA_ERR_INVALID, "gpa_residual_scale_bf16: 16-byte aligned rows and gamma required");
  const uint64_t total = (uint64_t)rows * (uint64_t)(cols / 8);
  if (total >= (1ull << 31))
    return fail(GPA_ERR_UNSUPPORTED, "gpa_residual_scale_bf16: more than 2^31 vectors");
  if (total == 0) return ok();
  const unsigned blocks = (unsigned)std::min<uint64_t>((total + 255) / 256, 148ull * 16);
  norm::residual_scale_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)x, x_stride, (const __nv_bfloat16*)y, y_stride,
      (const __nv_bfloat16*)gamma, (uint32_t)(cols / 8), (uint32_t)total, (__nv_bfloat16*)out,
      out_stride);
  return check_launch("gpa_residual_scale_bf16");
}

extern "C" int gpa_gelu_bf16(const void* x, int64_t n, void* out, void* stream) {
  if (n < 0 || n % 8)
    return fail(GPA_ERR_UNSUPPORTED, "gpa_gelu_bf16: element count must be a multiple of 8");
  if (!aligned16(x) || !aligned16(out)) return fail(GPA_ERR_INVALID, "gpa_gelu_bf16: 16-byte aligned buffers required");
  const int64_t nvec = n / 8;
  if (nvec == 0) return ok();
  const unsigned blocks = (unsigned)std::min<int64_t>((nvec + 255) / 256, 148ll * 32);
  norm::gelu_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>((const __nv_bfloat16*)x, (__nv_bfloat16*)out, nvec);
  return check_launch("gpa_gelu_bf16");
}
