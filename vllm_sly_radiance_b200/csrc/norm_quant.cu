// Fused producer kernels: every W4A8 linear consumes (e4m3 rows, fp32 per-row scale), and these
// kernels produce that pair straight from the residual stream / activations in one pass.
//
// Semantics (reference: sly/mxfp4/radiance_mxfp4_fp8.hip:1715-1730 add_rms_quant, :1941
// silu_mul_quant, :2079 gdn_norm_quant):
//   add_rms_quant : s = f32(x) + f32(res); res_out = bf16(s);
//                   n = bf16(s * rsqrt(mean(s^2) + eps) * (1 + w))           (Gemma weight)
//   silu_mul_quant: n = bf16(silu(g) * u)
//   gdn_norm_quant: n = bf16(bf16(o * rsqrt(mean_head(o^2) + eps) * w) * silu(z))  per 128-head
//   gate_mul_quant: n = bf16(o * sigmoid(gate))
//   then          : scale = max(amax|n| / 448, 1/(448*512)); q = e4m3_rne(n / scale)
// One CTA per row, the row held in registers between the reduction passes (8-element vectors).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace rad {
namespace nq {

constexpr int T = 256;   // threads per row
constexpr int V = 8;     // elements per vector

DEVI float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = (l < T / 32) ? red[l] : 0.f;
  return warp_sum(r);
}
DEVI float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = (l < T / 32) ? red[l] : 0.f;
  return warp_max(r);
}

DEVI void load8(const __nv_bfloat16* p, float (&f)[V]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
DEVI void load8(const float* p, float (&f)[V]) {
  float4 a = *reinterpret_cast<const float4*>(p);
  float4 b = *reinterpret_cast<const float4*>(p + 4);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}
DEVI void store8(__nv_bfloat16* p, const float (&f)[V]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}
DEVI void store8_fp8(uint8_t* p, const float (&f)[V], float inv) {
  uint2 u;
  uint16_t* h = reinterpret_cast<uint16_t*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = f32x2_to_e4m3x2(f[2 * i] * inv, f[2 * i + 1] * inv);
  *reinterpret_cast<uint2*>(p) = u;
}

// Final stage shared by all producers: values (already bf16-rounded) in registers.
template <int MAXV>
DEVI void quant_store(float (&vals)[MAXV][V], int nvec, uint8_t* qrow, float* scale_out, float* red) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * T;
    if (v < nvec) {
#pragma unroll
      for (int j = 0; j < V; ++j) amax = fmaxf(amax, fabsf(vals[i][j]));
    }
  }
  amax = block_max(amax, red);
  const float scale = fmaxf(amax / 448.f, 1.f / (448.f * 512.f));
  const float inv = 1.f / scale;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * T;
    if (v < nvec) store8_fp8(qrow + (size_t)v * V, vals[i], inv);
  }
  if (threadIdx.x == 0) *scale_out = scale;
}

template <int MAXV, bool QUANT>
__global__ void __launch_bounds__(T) add_rms_kernel(
    const __nv_bfloat16* __restrict__ x, int ldx, const __nv_bfloat16* __restrict__ res, int ldr,
    const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ res_out, int ldro,
    uint8_t* __restrict__ q, int ldq, float* __restrict__ scale, __nv_bfloat16* __restrict__ nout,
    int ldn, int H, float eps) {
  const int nvec = H / V;
  // the norm weight is a model constant: fetched before the dependency wait, off the critical path
  uint4 wraw[MAXV];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * T;
    if (v < nvec) wraw[i] = *reinterpret_cast<const uint4*>(w + v * V);
  }
  pdl_wait();     // inputs come from the preceding kernel
  pdl_trigger();
  __shared__ float red[T / 32];
  const int row = blockIdx.x;
  float vals[MAXV][V];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * T;
    if (v < nvec) {
      load8(x + (size_t)row * ldx + v * V, vals[i]);
      if (res) {
        float r[V];
        load8(res + (size_t)row * ldr + v * V, r);
#pragma unroll
        for (int j = 0; j < V; ++j) vals[i][j] += r[j];
      }
      if (res_out) store8(res_out + (size_t)row * ldro + v * V, vals[i]);
#pragma unroll
      for (int j = 0; j < V; ++j) ss += vals[i][j] * vals[i][j];
    }
  }
  ss = block_sum(ss, red);
  const float rs = rsqrtf(ss / (float)H + eps);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * T;
    if (v < nvec) {
      float wv[V];
      load8(reinterpret_cast<const __nv_bfloat16*>(&wraw[i]), wv);
#pragma unroll
      for (int j = 0; j < V; ++j) vals[i][j] = bf16_round(vals[i][j] * rs * (wv[j] + 1.f));
      if (nout) store8(nout + (size_t)row * ldn + v * V, vals[i]);
    }
  }
  if constexpr (QUANT) quant_store<MAXV>(vals, nvec, q + (size_t)row * ldq, scale + row, red);
}

template <int MAXV>
__global__ void __launch_bounds__(T) silu_mul_quant_kernel(const __nv_bfloat16* __restrict__ gu,
                                                           int ldg, int I, uint8_t* __restrict__ q,
                                                           int ldq, float* __restrict__ scale) {
  pdl_wait();     // inputs come from the preceding kernel
  pdl_trigger();
  __shared__ float red[T / 32];
  const int row = blockIdx.x;
  const int nvec = I / V;
  float vals[MAXV][V];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * T;
    if (v < nvec) {
      float g[V], u[V];
      load8(gu + (size_t)row * ldg + v * V, g);
      load8(gu + (size_t)row * ldg + I + v * V, u);
#pragma unroll
      for (int j = 0; j < V; ++j) vals[i][j] = bf16_round(g[j] / (1.f + __expf(-g[j])) * u[j]);
    }
  }
  quant_store<MAXV>(vals, nvec, q + (size_t)row * ldq, scale + row, red);
}

// o: [M, Hv*dv] (bf16 or fp32), z: strided bf16 view, per-head gated RMSNorm with weight [dv]
template <int MAXV, typename OT>
__global__ void __launch_bounds__(T) gdn_norm_quant_kernel(
    const OT* __restrict__ o, int ldo, const __nv_bfloat16* __restrict__ z, int ldz,
    const __nv_bfloat16* __restrict__ w, int D, int head_dim, float eps, uint8_t* __restrict__ q,
    int ldq, float* __restrict__ scale, __nv_bfloat16* __restrict__ nout, int ldn) {
  const int nvec = D / V;
  const int lanes_per_head = head_dim / V;     // 16 for head 128 (power of two <= 32)
  // the norm weight is a model constant: fetched before the dependency wait
  uint4 wraw[MAXV];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * T;
    if (v < nvec) wraw[i] = *reinterpret_cast<const uint4*>(w + (v * V) % head_dim);
  }
  pdl_wait();     // inputs come from the preceding kernel
  pdl_trigger();
  __shared__ float red[T / 32];
  const int row = blockIdx.x;
  float vals[MAXV][V];
  // z comes from an earlier kernel than o: both loads are issued before any reduction
  uint4 zraw[MAXV];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * T;
    if (v < nvec) {
      load8(o + (size_t)row * ldo + v * V, vals[i]);
      zraw[i] = *reinterpret_cast<const uint4*>(z + (size_t)row * ldz + v * V);
    }
  }
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * T;
    float ss = 0.f;
    if (v < nvec) {
#pragma unroll
      for (int j = 0; j < V; ++j) ss += vals[i][j] * vals[i][j];
    }
    // head reduction across the `lanes_per_head` consecutive threads owning this head
    for (int off = lanes_per_head / 2; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, off);
    if (v < nvec) {
      const float rs = rsqrtf(ss / (float)head_dim + eps);
      float wv[V], zv[V];
      load8(reinterpret_cast<const __nv_bfloat16*>(&wraw[i]), wv);
      load8(reinterpret_cast<const __nv_bfloat16*>(&zraw[i]), zv);
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const float nn = bf16_round(vals[i][j] * rs * wv[j]);
        vals[i][j] = bf16_round(nn * (zv[j] / (1.f + __expf(-zv[j]))));
      }
      if (nout) store8(nout + (size_t)row * ldn + v * V, vals[i]);
    }
  }
  if (q) quant_store<MAXV>(vals, nvec, q + (size_t)row * ldq, scale + row, red);
}

template <int MAXV>
__global__ void __launch_bounds__(T) gate_mul_quant_kernel(
    const __nv_bfloat16* __restrict__ a, int lda, const __nv_bfloat16* __restrict__ gate, int ldg,
    int head_dim, int gate_head_stride, int D, uint8_t* __restrict__ q, int ldq,
    float* __restrict__ scale, __nv_bfloat16* __restrict__ nout, int ldn) {
  pdl_wait();     // inputs come from the preceding kernel
  pdl_trigger();
  __shared__ float red[T / 32];
  const int row = blockIdx.x;
  const int nvec = D / V;
  float vals[MAXV][V];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * T;
    if (v < nvec) {
      float gv[V];
      load8(a + (size_t)row * lda + v * V, vals[i]);
      const int e = v * V;
      const int h = e / head_dim, c = e % head_dim;
      load8(gate + (size_t)row * ldg + (size_t)h * gate_head_stride + c, gv);
#pragma unroll
      for (int j = 0; j < V; ++j) vals[i][j] = bf16_round(vals[i][j] / (1.f + __expf(-gv[j])));
      if (nout) store8(nout + (size_t)row * ldn + v * V, vals[i]);
    }
  }
  if (q) quant_store<MAXV>(vals, nvec, q + (size_t)row * ldq, scale + row, red);
}

template <int MAXV>
__global__ void __launch_bounds__(T) quant_rows_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                                                       int D, uint8_t* __restrict__ q, int ldq,
                                                       float* __restrict__ scale) {
  pdl_wait();     // inputs come from the preceding kernel
  pdl_trigger();
  __shared__ float red[T / 32];
  const int row = blockIdx.x;
  const int nvec = D / V;
  float vals[MAXV][V];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * T;
    if (v < nvec) load8(x + (size_t)row * ldx + v * V, vals[i]);
  }
  quant_store<MAXV>(vals, nvec, q + (size_t)row * ldq, scale + row, red);
}

#define DISPATCH_MAXV(NVEC, ...)                                   \
  do {                                                             \
    const int _nv = (NVEC);                                        \
    if (_nv <= T) { constexpr int MAXV = 1; __VA_ARGS__; }         \
    else if (_nv <= 2 * T) { constexpr int MAXV = 2; __VA_ARGS__; } \
    else if (_nv <= 3 * T) { constexpr int MAXV = 3; __VA_ARGS__; } \
    else if (_nv <= 5 * T) { constexpr int MAXV = 5; __VA_ARGS__; } \
    else if (_nv <= 9 * T) { constexpr int MAXV = 9; __VA_ARGS__; } \
    else if (_nv <= 13 * T) { constexpr int MAXV = 13; __VA_ARGS__; } \
    else TORCH_CHECK(false, "row too long for producer kernel");   \
  } while (0)

static inline const __nv_bfloat16* bf(const torch::Tensor& t) {
  return t.defined() && t.numel() ? reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()) : nullptr;
}
static inline __nv_bfloat16* bfm(const torch::Tensor& t) {
  return t.defined() && t.numel() ? reinterpret_cast<__nv_bfloat16*>(t.data_ptr()) : nullptr;
}

// The producers move rows with 16-byte vector loads / stores (8-byte for the e4m3 output): a
// tensor whose base or row stride breaks that alignment is rejected here instead of faulting.
static inline void check_vec(const torch::Tensor& t, const char* what, int align = 16) {
  if (!t.defined() || t.numel() == 0) return;
  const int64_t es = t.element_size();
  TORCH_CHECK(t.stride(-1) == 1 && reinterpret_cast<uintptr_t>(t.data_ptr()) % align == 0 &&
                  (t.dim() < 2 || (t.stride(0) * es) % align == 0),
              what, ": vector access needs a ", align, "-byte aligned base and row stride");
}

}  // namespace nq

// x [M,H] bf16; residual (optional, may alias res_out); q fp8 [M,H] / scale [M] (optional);
// nout bf16 (optional normalized output)
void add_rms_quant(torch::Tensor x, torch::Tensor residual, torch::Tensor weight,
                   torch::Tensor res_out, torch::Tensor q, torch::Tensor scale,
                   torch::Tensor nout, double eps) {
  using namespace nq;
  const int M = x.size(0), H = x.size(1);
  TORCH_CHECK(H % V == 0 && x.stride(1) == 1, "add_rms_quant: H % 8 and row-major");
  check_vec(x, "add_rms_quant x");
  check_vec(weight, "add_rms_quant weight");
  check_vec(residual, "add_rms_quant residual");
  check_vec(res_out, "add_rms_quant res_out");
  check_vec(nout, "add_rms_quant nout");
  check_vec(q, "add_rms_quant q", 8);
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const bool quant = q.defined() && q.numel();
  DISPATCH_MAXV(H / V, {
    if (quant)
C10_CUDA_CHECK(launch_pdl((add_rms_kernel<MAXV, true>), dim3(M), dim3(T), 0, stream, 
          bf(x), x.stride(0), bf(residual), residual.defined() && residual.numel() ? residual.stride(0) : 0,
          bf(weight), bfm(res_out), res_out.defined() && res_out.numel() ? res_out.stride(0) : 0,
          (uint8_t*)q.data_ptr(), q.stride(0), scale.data_ptr<float>(), bfm(nout),
          nout.defined() && nout.numel() ? nout.stride(0) : 0, H, (float)eps));
    else
C10_CUDA_CHECK(launch_pdl((add_rms_kernel<MAXV, false>), dim3(M), dim3(T), 0, stream, 
          bf(x), x.stride(0), bf(residual), residual.defined() && residual.numel() ? residual.stride(0) : 0,
          bf(weight), bfm(res_out), res_out.defined() && res_out.numel() ? res_out.stride(0) : 0,
          nullptr, 0, nullptr, bfm(nout), nout.defined() && nout.numel() ? nout.stride(0) : 0, H,
          (float)eps));
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void silu_mul_quant(torch::Tensor gate_up, torch::Tensor q, torch::Tensor scale) {
  using namespace nq;
  const int M = gate_up.size(0), I = gate_up.size(1) / 2;
  TORCH_CHECK(I % V == 0 && gate_up.stride(1) == 1, "silu_mul_quant: I % 8");
  check_vec(gate_up, "silu_mul_quant gate_up");
  check_vec(q, "silu_mul_quant q", 8);
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(gate_up.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  DISPATCH_MAXV(I / V, {
C10_CUDA_CHECK(launch_pdl((silu_mul_quant_kernel<MAXV>), dim3(M), dim3(T), 0, stream, bf(gate_up), gate_up.stride(0), I,
                                                      (uint8_t*)q.data_ptr(), q.stride(0),
                                                      scale.data_ptr<float>()));
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gdn_norm_quant(torch::Tensor o, torch::Tensor z, torch::Tensor weight, int64_t head_dim,
                    double eps, torch::Tensor q, torch::Tensor scale, torch::Tensor nout) {
  using namespace nq;
  const int M = o.size(0), D = o.size(1);
  TORCH_CHECK(D % V == 0 && head_dim % V == 0 && (head_dim / V) <= 32 &&
                  ((head_dim / V) & (head_dim / V - 1)) == 0,
              "gdn_norm_quant: unsupported head_dim");
  check_vec(o, "gdn_norm_quant o");
  check_vec(weight, "gdn_norm_quant weight");
  check_vec(z, "gdn_norm_quant z");
  check_vec(q, "gdn_norm_quant q", 8);
  check_vec(nout, "gdn_norm_quant nout");
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(o.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  uint8_t* qp = q.defined() && q.numel() ? (uint8_t*)q.data_ptr() : nullptr;
  float* sp = qp ? scale.data_ptr<float>() : nullptr;
  const int ldq = qp ? q.stride(0) : 0;
  const int ldn = nout.defined() && nout.numel() ? nout.stride(0) : 0;
  DISPATCH_MAXV(D / V, {
    if (o.scalar_type() == at::kFloat)
C10_CUDA_CHECK(launch_pdl((gdn_norm_quant_kernel<MAXV, float>), dim3(M), dim3(T), 0, stream, 
          o.data_ptr<float>(), o.stride(0), bf(z), z.stride(0), bf(weight), D, head_dim, (float)eps,
          qp, ldq, sp, bfm(nout), ldn));
    else
C10_CUDA_CHECK(launch_pdl((gdn_norm_quant_kernel<MAXV, __nv_bfloat16>), dim3(M), dim3(T), 0, stream, 
          bf(o), o.stride(0), bf(z), z.stride(0), bf(weight), D, head_dim, (float)eps, qp, ldq, sp,
          bfm(nout), ldn));
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// a [M, H*hd] bf16; gate = bf16 view with row stride ldg, head h at column h*gate_head_stride
void gate_mul_quant(torch::Tensor a, torch::Tensor gate, int64_t head_dim, int64_t gate_head_stride,
                    torch::Tensor q, torch::Tensor scale, torch::Tensor nout) {
  using namespace nq;
  const int M = a.size(0), D = a.size(1);
  TORCH_CHECK(D % V == 0 && head_dim % V == 0 && gate_head_stride % V == 0,
              "gate_mul_quant: dims % 8");
  check_vec(a, "gate_mul_quant a");
  check_vec(gate, "gate_mul_quant gate");
  check_vec(q, "gate_mul_quant q", 8);
  check_vec(nout, "gate_mul_quant nout");
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(a.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  uint8_t* qp = q.defined() && q.numel() ? (uint8_t*)q.data_ptr() : nullptr;
  float* sp = qp ? scale.data_ptr<float>() : nullptr;
  const int ldq = qp ? q.stride(0) : 0;
  const int ldn = nout.defined() && nout.numel() ? nout.stride(0) : 0;
  DISPATCH_MAXV(D / V, {
C10_CUDA_CHECK(launch_pdl((gate_mul_quant_kernel<MAXV>), dim3(M), dim3(T), 0, stream, bf(a), a.stride(0), bf(gate), gate.stride(0),
                                                     head_dim, gate_head_stride, D, qp, ldq, sp,
                                                     bfm(nout), ldn));
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void quant_fp8_rows(torch::Tensor x, torch::Tensor q, torch::Tensor scale) {
  using namespace nq;
  const int M = x.size(0), D = x.size(1);
  TORCH_CHECK(D % V == 0, "quant_fp8_rows: D % 8");
  check_vec(x, "quant_fp8_rows x");
  check_vec(q, "quant_fp8_rows q", 8);
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  DISPATCH_MAXV(D / V, {
C10_CUDA_CHECK(launch_pdl((quant_rows_kernel<MAXV>), dim3(M), dim3(T), 0, stream, bf(x), x.stride(0), D, (uint8_t*)q.data_ptr(),
                                                 q.stride(0), scale.data_ptr<float>()));
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace rad
