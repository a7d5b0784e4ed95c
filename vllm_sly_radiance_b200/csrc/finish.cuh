// Row finishers: the producer that follows a decode kernel (residual add + RMSNorm(1 + w) + e4m3,
// or SiLU(g) * u + e4m3) run by the one CTA that completes the producing kernel's last output
// tile, instead of a separate launch.  The numerics are those of the stand-alone producers
// (norm_quant.cu):
//   norm: s = f32(x) + f32(res); res_out = bf16(s); y = bf16(s * rsqrt(mean(s^2) + eps) * (1 + w))
//   silu: y = bf16(silu(g) * u) with x = [g | u]
//   then  scale = max(amax|y| / 448, 1 / (448 * 512)); q = e4m3_rne(y / scale)
// Reference behaviour: the fused producers of sly/mxfp4/radiance_mxfp4_fp8.hip (:1835
// add_rms_quant, :1941 silu_mul_quant) and the decode GEMM's in-kernel last-block reduction
// (:1251-1343), which this combines: the last block finishes the row instead of a new kernel.
#pragma once

#include "common.cuh"

namespace rad {

enum FinMode : int { kFinNone = 0, kFinNorm = 1, kFinSilu = 2 };

struct FinArgs {
  const __nv_bfloat16* res;   // norm: residual in (nullable)
  int ldr;
  const __nv_bfloat16* w;     // norm: weight of the Gemma (1 + w) RMSNorm
  __nv_bfloat16* res_out;     // norm: new residual stream (nullable)
  int ldro;
  uint8_t* q;                 // e4m3 rows
  int ldq;
  float* scale;               // per-row scale
  float eps;
};

template <int NT>
DEVI float fin_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) r += red[i];
  return r;
}
template <int NT>
DEVI float fin_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) r = fmaxf(r, red[i]);
  return r;
}

DEVI void fin_ld8_cg(const __nv_bfloat16* p, float (&f)[8]) {
  // written by other CTAs of this grid: read through L2
  const uint4 u = __ldcg(reinterpret_cast<const uint4*>(p));
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
DEVI void fin_ld8(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
DEVI void fin_st8(__nv_bfloat16* p, const float (&f)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

// e4m3 quantisation of the bf16-valued row in buf[0, H) (smem), amax already known
template <int NT>
DEVI void fin_quant_store(const float* buf, int H, float amax, uint8_t* qrow, float* scale_out) {
  const float scale = fmaxf(amax / 448.f, 1.f / (448.f * 512.f));
  const float inv = 1.f / scale;
  for (int v = threadIdx.x; v < H / 8; v += NT) {
    uint2 u;
    uint16_t* h = reinterpret_cast<uint16_t*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = f32x2_to_e4m3x2(buf[v * 8 + 2 * i] * inv, buf[v * 8 + 2 * i + 1] * inv);
    *reinterpret_cast<uint2*>(qrow + (size_t)v * 8) = u;
  }
  if (threadIdx.x == 0) *scale_out = scale;
}

// Row m of x ([., H] bf16, row stride ldx; written by this grid) -> e4m3 row + scale.  All NT
// threads of the CTA call this; buf holds >= H (norm) or >= H / 2 (silu) floats of shared memory.
template <int NT, int MODE>
DEVI void finish_row(const FinArgs& f, const __nv_bfloat16* x, int ldx, int H, int m, float* buf,
                     float* red) {
  const __nv_bfloat16* xr = x + (size_t)m * ldx;
  if constexpr (MODE == kFinNorm) {
    float ss = 0.f;
    for (int v = threadIdx.x; v < H / 8; v += NT) {
      float s[8];
      fin_ld8_cg(xr + v * 8, s);
      if (f.res) {
        float r[8];
        fin_ld8(f.res + (size_t)m * f.ldr + v * 8, r);
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j] += r[j];
      }
      if (f.res_out) fin_st8(f.res_out + (size_t)m * f.ldro + v * 8, s);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        ss += s[j] * s[j];
        buf[v * 8 + j] = s[j];
      }
    }
    ss = fin_sum<NT>(ss, red);
    const float rs = rsqrtf(ss / (float)H + f.eps);
    float amax = 0.f;
    for (int v = threadIdx.x; v < H / 8; v += NT) {
      float wv[8];
      fin_ld8(f.w + v * 8, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float y = bf16_round(buf[v * 8 + j] * rs * (wv[j] + 1.f));
        buf[v * 8 + j] = y;
        amax = fmaxf(amax, fabsf(y));
      }
    }
    amax = fin_max<NT>(amax, red);
    fin_quant_store<NT>(buf, H, amax, f.q + (size_t)m * f.ldq, f.scale + m);
  } else {
    const int I = H / 2;
    float amax = 0.f;
    for (int v = threadIdx.x; v < I / 8; v += NT) {
      float g[8], u[8];
      fin_ld8_cg(xr + v * 8, g);
      fin_ld8_cg(xr + I + v * 8, u);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float y = bf16_round(g[j] / (1.f + __expf(-g[j])) * u[j]);
        buf[v * 8 + j] = y;
        amax = fmaxf(amax, fabsf(y));
      }
    }
    amax = fin_max<NT>(amax, red);
    fin_quant_store<NT>(buf, I, amax, f.q + (size_t)m * f.ldq, f.scale + m);
  }
  __syncthreads();   // buf is reused by the next row
}

}  // namespace rad
