// Bilinear resize of the DPT head's feature maps (align_corners=True), fused
// with the bf16 cast the following autocast convolution applies to its input,
// and optionally with the head's fp32 positional-embedding add.
//
// Reference: heads/dpt_head.py custom_interpolate (F.interpolate, bilinear,
// align_corners=True) feeding out_conv / output_conv2, and _apply_pos_embed
// (x + pos_embed) before output_conv2.  Under bf16 autocast the interpolation
// runs in fp32 and the convolution rounds its input to bf16; this kernel
// computes the same fp32 value (torch's source-index and lambda arithmetic)
// and writes the bf16 the convolution would have received, in one pass
// instead of an fp32 resize, an fp32 add and a cast.
//
// Layout: channels-last ([N, H, W, C] in memory, C contiguous) in and out; one
// thread per output pixel and 8 channels.  The input may be fp32 or bf16 (a
// bf16 map is exactly representable in the fp32 the resize computes in).
#include "common.cuh"
#include "capi_util.h"

namespace gpa {
namespace dpt {

__device__ __forceinline__ void load8(const float* p, float* v) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* v) {
  const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
  const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 f = __bfloat1622float2(e[k]);
    v[2 * k] = f.x;
    v[2 * k + 1] = f.y;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) upsample_bilinear_kernel(
    const T* __restrict__ x, int64_t xsn, int64_t xsh, int64_t xsw, int C, int H, int W,
    const float* __restrict__ add, int64_t ash, int64_t asw, int round_first,
    __nv_bfloat16* __restrict__ out, int64_t osn, int64_t osh, int64_t osw, int OH, int OW, float rh,
    float rw, int64_t total) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int c8 = C / 8;
  const int cg = (int)(i % c8);
  int64_t rest = i / c8;
  const int ox = (int)(rest % OW);
  rest /= OW;
  const int oy = (int)(rest % OH);
  const int64_t n = rest / OH;
  // source index and weights as torch computes them for align_corners=True
  const float h1r = rh * (float)oy;
  const int h1 = (int)h1r;
  const int h1p = h1 < H - 1 ? 1 : 0;
  const float h1l = h1r - (float)h1;
  const float h0l = 1.0f - h1l;
  const float w1r = rw * (float)ox;
  const int w1 = (int)w1r;
  const int w1p = w1 < W - 1 ? 1 : 0;
  const float w1l = w1r - (float)w1;
  const float w0l = 1.0f - w1l;
  const T* base = x + n * xsn + (int64_t)h1 * xsh + (int64_t)w1 * xsw + cg * 8;
  float a[8], b[8], c[8], d[8];
  load8(base, a);
  load8(base + w1p * xsw, b);
  load8(base + h1p * xsh, c);
  load8(base + h1p * xsh + w1p * xsw, d);
  float v[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) v[k] = h0l * (w0l * a[k] + w1l * b[k]) + h1l * (w0l * c[k] + w1l * d[k]);
  if (add) {
    float e[8];
    load8(add + (int64_t)oy * ash + (int64_t)ox * asw + cg * 8, e);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      // round_first: the resize result was a bf16 tensor before the fp32 add
      const float r = round_first ? __bfloat162float(__float2bfloat16_rn(v[k])) : v[k];
      v[k] = __fadd_rn(r, e[k]);
    }
  }
  uint4 raw;
  __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
  for (int k = 0; k < 4; ++k) o2[k] = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
  *reinterpret_cast<uint4*>(out + n * osn + (int64_t)oy * osh + (int64_t)ox * osw + cg * 8) = raw;
}

}  // namespace dpt
}  // namespace gpa

using namespace gpa;

extern "C" int gpa_upsample_bilinear_bf16(const void* x, int x_dtype, int n, int c, int h, int w,
                                          int64_t x_sn, int64_t x_sh, int64_t x_sw, const float* add,
                                          int64_t add_sh, int64_t add_sw, int round_first, int out_h,
                                          int out_w, void* out, int64_t out_sn, int64_t out_sh,
                                          int64_t out_sw, void* stream) {
  if (x_dtype != GPA_DTYPE_F32 && x_dtype != GPA_DTYPE_BF16)
    return fail(GPA_ERR_INVALID, "gpa_upsample_bilinear_bf16: input dtype must be f32 or bf16");
  const int64_t xalign = x_dtype == GPA_DTYPE_F32 ? 4 : 8;   // elements per 16 bytes
  if (n < 0 || c <= 0 || h <= 0 || w <= 0 || out_h <= 0 || out_w <= 0)
    return fail(GPA_ERR_INVALID, "gpa_upsample_bilinear_bf16: bad sizes");
  if (c % 8)
    return fail(GPA_ERR_UNSUPPORTED, "gpa_upsample_bilinear_bf16: channels must be a multiple of 8");
  if (!aligned16(x) || !aligned16(out) || (add && !aligned16(add)) || x_sn % xalign || x_sh % xalign ||
      x_sw % xalign ||
      (add && (add_sh % 4 || add_sw % 4)) || out_sn % 8 || out_sh % 8 || out_sw % 8)
    return fail(GPA_ERR_INVALID,
                "gpa_upsample_bilinear_bf16: channels-last rows with 16-byte aligned pixels required");
  const int64_t total = (int64_t)n * out_h * out_w * (c / 8);
  if (total == 0) return ok();
  // align_corners=True: scale = (in - 1) / (out - 1), 0 for a single output row
  const float rh = out_h > 1 ? (float)(h - 1) / (float)(out_h - 1) : 0.0f;
  const float rw = out_w > 1 ? (float)(w - 1) / (float)(out_w - 1) : 0.0f;
  const int64_t blocks = (total + 255) / 256;
  if (blocks > 0x7fffffffll) return fail(GPA_ERR_UNSUPPORTED, "gpa_upsample_bilinear_bf16: too large");
  cudaStream_t st = (cudaStream_t)stream;
  if (x_dtype == GPA_DTYPE_F32)
    dpt::upsample_bilinear_kernel<float><<<(unsigned)blocks, 256, 0, st>>>(
        (const float*)x, x_sn, x_sh, x_sw, c, h, w, add, add_sh, add_sw, round_first,
        (__nv_bfloat16*)out, out_sn, out_sh, out_sw, out_h, out_w, rh, rw, total);
  else
    dpt::upsample_bilinear_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, st>>>(
        (const __nv_bfloat16*)x, x_sn, x_sh, x_sw, c, h, w, add, add_sh, add_sw, round_first,
        (__nv_bfloat16*)out, out_sn, out_sh, out_sw, out_h, out_w, rh, rw, total);
  return check_launch("gpa_upsample_bilinear_bf16");
}

// ---------------------------------------------------------------------------
// Convolution bias, ReLU and residual of the DPT head's convolutions, in one
// pass over a channels-last bf16 map (replaces the bias add torch issues after
// each cuDNN convolution, the ReLU of ResidualConvUnit and its skip add;
// heads/dpt_head.py ResidualConvUnit, FeatureFusionBlock):
//   t   = bf16(y + bias[c])            the conv's bias add (bf16 tensors, fp32 math)
//   t   = relu(t)                      when relu != 0
//   out = bf16(t + res)                when res != NULL (the residual add)
// Each step rounds as the torch op it replaces, so the result is bit-exact.
// y, res, out: [N, H, W, C] contiguous bf16 (channels-last), C % 8 == 0; out
// may be y.  One thread per 8 channels of a pixel.
// ---------------------------------------------------------------------------
namespace gpa {
namespace dpt {
__global__ void __launch_bounds__(256) bias_act_kernel(const __nv_bfloat16* __restrict__ y,
                                                       const __nv_bfloat16* __restrict__ bias,
                                                       const __nv_bfloat16* __restrict__ res, int c,
                                                       int64_t groups, int relu, __nv_bfloat16* out) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= groups) return;
  const int c0 = (int)((g * 8) % c);
  float v[8], b[8];
  load8(y + g * 8, v);
  load8(bias + c0, b);
  float r[8];
  if (res) load8(res + g * 8, r);
  uint4 pk;
  __nv_bfloat162* e = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float t0 = __bfloat162float(__float2bfloat16_rn(v[2 * k] + b[2 * k]));
    float t1 = __bfloat162float(__float2bfloat16_rn(v[2 * k + 1] + b[2 * k + 1]));
    if (relu) {
      t0 = fmaxf(t0, 0.0f);
      t1 = fmaxf(t1, 0.0f);
    }
    if (res) {
      t0 += r[2 * k];
      t1 += r[2 * k + 1];
    }
    e[k] = __floats2bfloat162_rn(t0, t1);
  }
  *reinterpret_cast<uint4*>(out + g * 8) = pk;
}
}  // namespace dpt
}  // namespace gpa

extern "C" int gpa_bias_act_bf16(const void* y, const void* bias, const void* res, int64_t pixels, int c,
                                 int relu, void* out, void* stream) {
  if (pixels < 0 || c <= 0 || c % 8)
    return fail(GPA_ERR_INVALID, "gpa_bias_act_bf16: channels must be a positive multiple of 8");
  if (!y || !bias || !out || !aligned16(y) || !aligned16(bias) || !aligned16(out) || (res && !aligned16(res)))
    return fail(GPA_ERR_INVALID, "gpa_bias_act_bf16: null or unaligned pointer");
  const int64_t groups = pixels * (c / 8);
  if (groups == 0) return ok();
  const int64_t blocks = (groups + 255) / 256;
  if (blocks > 0x7fffffffll) return fail(GPA_ERR_UNSUPPORTED, "gpa_bias_act_bf16: too large");
  dpt::bias_act_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)y, (const __nv_bfloat16*)bias, (const __nv_bfloat16*)res, c, groups, relu,
      (__nv_bfloat16*)out);
  return check_launch("gpa_bias_act_bf16");
}

