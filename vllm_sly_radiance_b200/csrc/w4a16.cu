// W4A16 linear: int4 weights (g128, asymmetric: per group fp16 scale + uint8 zero point) with
// bf16 activations.
//
// Reference behaviour: the W4A16 split-K Triton GEMM (sly/patch_w4a16_tiles.py:226-420) and the
// HIP wvSplitK_int4_g path used for the DFlash2 drafter, INT4 targets and the int4 lm_head
// (sly/mxfp4/radiance_lmhead_int4.py): y[m, n] = sum_k x[m, k] * (q[n, k] - z[n, k/128]) *
// s[n, k/128].
//
// B200 design (decode, M <= 8 rows): the kernel is a weight stream, so the work per weight byte
// must be a handful of instructions.  The weight is re-laid at load time into tensor-core
// fragment order (quant/int4.py ``mma_tile``): one 16-byte load gives a lane its mma.m16n8k16
// A fragments for four k-steps of a 16-row tile; a nibble pair becomes the exact bf16x2
// (128 + q) with one shift and one mask-or against 0x4300 (= 128.0) -- no float arithmetic
// per weight (a bf16x2 subtract is not a native instruction here and ran through conversions);
// the tensor core does the dot products in fp32 against the activations (the B operand, tokens
// as the n dimension); per 128-column group the zero point comes off as (128 + z) * sum(x),
// sum(x) taken by one more MMA against an all-ones A, and the scale multiplies the fp32 group
// partial once.  Four warps of a CTA split K for TW row tiles and a thread-block cluster along y
// splits it further; each warp streams its slice through a ring of shared-memory stages filled
// by bulk copies (cp.async.bulk + mbarrier, bounded waits).  Partials meet in shared memory and
// then over distributed shared memory.  The first stages are fetched before the
// programmatic-dependency wait, overlapping the predecessor's tail.  Prefill (larger M) expands
// row blocks to bf16 (w4a16_dequant_kernel) for a library GEMM.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdlib>

#include "common.cuh"

namespace rad {
namespace w4 {

constexpr int G = 128;          // quantisation group (two 64-column blocks)
constexpr int WARPS = 4;
constexpr int MAXM = 8;
constexpr int MAXC = 8;         // cluster K-split

DEVI void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// one pipeline stage of a warp: one group (128 columns = two 64-column blocks) of TW tiles
template <int TW>
struct Stage {
  uint4 w[TW][2][32];   // A fragments: [tile][block][lane] -> 4 steps
  uint2 sz[TW][8];      // fp16x2 scales, bf16x2 (128 + zero) of rows (g, g + 8)
};

DEVI void load_x(uint4 (&xv)[2][2], const __nv_bfloat16* __restrict__ x, int ldx, int Mr, int gi,
                 int lane) {
  const int n = lane >> 2, t = lane & 3;
#pragma unroll
  for (int b = 0; b < 2; ++b)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      xv[b][h] = make_uint4(0, 0, 0, 0);
      if (n < Mr)
        xv[b][h] = __ldg(reinterpret_cast<const uint4*>(x + (size_t)n * ldx + gi * G + b * 64 +
                                                        t * 16) + h);
    }
}

template <int TW>
DEVI void compute(const Stage<TW>& st, const uint4 (&xv)[2][2], float (&acc)[TW][4], int lane) {
  const uint32_t xr[2][8] = {{xv[0][0].x, xv[0][0].y, xv[0][0].z, xv[0][0].w,
                              xv[0][1].x, xv[0][1].y, xv[0][1].z, xv[0][1].w},
                             {xv[1][0].x, xv[1][0].y, xv[1][0].z, xv[1][0].w,
                              xv[1][1].x, xv[1][1].y, xv[1][1].z, xv[1][1].w}};
  // independent accumulator chains (one per 64-column block) keep several MMAs in flight
  float xs[2][4] = {};
  {
    const uint32_t ones[4] = {0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u};
#pragma unroll
    for (int s = 0; s < 4; ++s)
#pragma unroll
      for (int b = 0; b < 2; ++b) mma_bf16(xs[b], ones, xr[b][2 * s], xr[b][2 * s + 1]);
  }
  float c[TW][2][4] = {};
#pragma unroll
  for (int s = 0; s < 4; ++s)
#pragma unroll
    for (int i = 0; i < TW; ++i)
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        const uint4 w4 = st.w[i][b][lane];
        const uint32_t q = s == 0 ? w4.x : s == 1 ? w4.y : s == 2 ? w4.z : w4.w;
        const uint32_t a[4] = {(q & 0x000F000Fu) | 0x43004300u,
                               ((q >> 4) & 0x000F000Fu) | 0x43004300u,
                               ((q >> 8) & 0x000F000Fu) | 0x43004300u,
                               ((q >> 12) & 0x000F000Fu) | 0x43004300u};
        mma_bf16(c[i][b], a, xr[b][2 * s], xr[b][2 * s + 1]);
      }
#pragma unroll
  for (int i = 0; i < TW; ++i) {
    const uint2 szv = st.sz[i][lane >> 2];
    const float2 sc = __half22float2(*reinterpret_cast<const __half2*>(&szv.x));
    const float zl = __uint_as_float(szv.y << 16);             // 128 + z[g]
    const float zh = __uint_as_float(szv.y & 0xFFFF0000u);     // 128 + z[g + 8]
    const float x0 = xs[0][0] + xs[1][0], x1 = xs[0][1] + xs[1][1];
    acc[i][0] += sc.x * fmaf(-zl, x0, c[i][0][0] + c[i][1][0]);
    acc[i][1] += sc.x * fmaf(-zl, x1, c[i][0][1] + c[i][1][1]);
    acc[i][2] += sc.y * fmaf(-zh, x0, c[i][0][2] + c[i][1][2]);
    acc[i][3] += sc.y * fmaf(-zh, x1, c[i][0][3] + c[i][1][3]);
  }
}

// grid (ceil(tiles / TW), C), cluster (1, C, 1), 128 threads.  Warp w of cluster CTA r takes the
// K slice r * 4 + w of C * 4 and streams it through a private ring of S shared-memory stages
// filled by bulk copies (one lane issues them, an mbarrier per stage counts the bytes).
template <int TW, int S>
__global__ void __launch_bounds__(32 * WARPS) w4a16_gemv_kernel(
    const __nv_bfloat16* __restrict__ x, int ldx, const uint4* __restrict__ wq,
    const uint2* __restrict__ sz, int N, int K, int Mr, __nv_bfloat16* __restrict__ out, int ldo,
    int* __restrict__ status) {
  __shared__ __align__(128) Stage<TW> ring[WARPS][S];
  __shared__ __align__(8) uint64_t full[WARPS][S];
  __shared__ float red[WARPS][TW][4][32];
  __shared__ __align__(16) float fin[TW * 16 * MAXM];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = (N + 15) / 16, KB = K / 64, NG = K / G;
  const int t0 = blockIdx.x * TW;
  const int C = gridDim.y;
  const int ks = blockIdx.y * WARPS + warp, KS = C * WARPS;
  const int g0 = ks * NG / KS, g1 = (ks + 1) * NG / KS;
  constexpr uint32_t kStageBytes = TW * (2 * 32 * 16 + 8 * 8);

  auto issue = [&](int slot, int gi) {
    mbar_arrive_expect_tx(&full[warp][slot], kStageBytes);
#pragma unroll
    for (int i = 0; i < TW; ++i) {
      const int T = min(t0 + i, ntiles - 1);
      bulk_load(&ring[warp][slot].w[i][0][0], wq + ((size_t)T * KB + 2 * gi) * 32, 2 * 32 * 16,
                &full[warp][slot]);
      bulk_load(&ring[warp][slot].sz[i][0], sz + ((size_t)T * NG + gi) * 8, 8 * 8,
                &full[warp][slot]);
    }
  };
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < S; ++s) mbar_init(&full[warp][s], 1);
    fence_mbar_init();
    // weights are constant: the first stages stream in before the dependency wait
    for (int s = 0; s < S && g0 + s < g1; ++s) issue(s, g0 + s);
  }
  __syncwarp();
  pdl_wait();     // activations come from the preceding kernel
  pdl_trigger();

  float acc[TW][4];
#pragma unroll
  for (int i = 0; i < TW; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  bool ok = true;
  int issued = min(S, g1 - g0), j = 0;
  // the activations of group j + 1 are loaded while group j computes (an L2 round trip per
  // group would otherwise sit on every warp's critical path)
  uint4 xv[2][2];
  if (g0 < g1) load_x(xv, x, ldx, Mr, g0, lane);
  for (; j < g1 - g0 && ok; ++j) {
    const int slot = j % S;
    uint4 xn[2][2];
    if (j + 1 < g1 - g0) load_x(xn, x, ldx, Mr, g0 + j + 1, lane);
    ok = mbar_wait(&full[warp][slot], (j / S) & 1, status);
    if (!ok) break;
    compute(ring[warp][slot], xv, acc, lane);
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int h = 0; h < 2; ++h) xv[b][h] = xn[b][h];
    __syncwarp();
    if (j + S < g1 - g0) {
      if (lane == 0) {
        fence_proxy_async();      // this warp's reads of the slot precede the copy into it
        issue(slot, g0 + j + S);
      }
      ++issued;
    }
  }
  // after a timed-out wait, give the copies still in flight a bounded time to land before the
  // shared memory is released
  for (int jj = ok ? issued : j; jj < issued; ++jj)
    mbar_wait(&full[warp][jj % S], (jj / S) & 1, nullptr);
  // D fragment: acc[i][0..1] = rows g, tokens 2t, 2t+1; acc[i][2..3] = row g + 8
#pragma unroll
  for (int i = 0; i < TW; ++i)
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) red[warp][i][jj][lane] = acc[i][jj];
  __syncthreads();
  for (int e = threadIdx.x; e < TW * 128; e += blockDim.x) {
    const int i = e >> 7, jj = (e >> 5) & 3, l = e & 31;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) v += red[w][i][jj][l];
    const int row = (l >> 2) + ((jj & 2) ? 8 : 0), tok = 2 * (l & 3) + (jj & 1);
    fin[(i * 16 + row) * MAXM + tok] = v;
  }
  if (C > 1) {
    cluster_sync();
    if (blockIdx.y == 0) {
      const uint32_t base = smem_u32(fin);
      for (int e = threadIdx.x; e < TW * 16 * MAXM / 4; e += blockDim.x) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < C; ++r) {
          const float4 u = ld_dsmem_f4(mapa_shared(base + e * 16, r));
          v.x += u.x; v.y += u.y; v.z += u.z; v.w += u.w;
        }
        const int row = e / (MAXM / 4), tk = (e % (MAXM / 4)) * 4;
        const int n = t0 * 16 + row;
        const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (n < N && tk + q < Mr) out[(size_t)(tk + q) * ldo + n] = __float2bfloat16_rn(vv[q]);
      }
    }
    cluster_sync();     // peers' shared memory stays alive until CTA 0 has read it
  } else {
    __syncthreads();
    for (int e = threadIdx.x; e < TW * 16 * MAXM; e += blockDim.x) {
      const int row = e / MAXM, tk = e % MAXM;
      const int n = t0 * 16 + row;
      if (n < N && tk < Mr) out[(size_t)tk * ldo + n] = __float2bfloat16_rn(fin[e]);
    }
  }
}

// rows [n0, n0 + rows) (n0 % 16 == 0) of the tiled weight -> bf16 [rows, K]; one thread per
// (tile, 64-column block, lane) expands 32 weights into two 32-byte row segments
__global__ void w4a16_dequant_kernel(const uint4* __restrict__ wq, const uint2* __restrict__ sz,
                                     int K, int n0, int rows, __nv_bfloat16* __restrict__ out) {
  const int KB = K / 64, NG = K / G;
  const int T0 = n0 / 16, nt = (rows + 15) / 16;
  const size_t total = (size_t)nt * KB * 32;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int lane = (int)(idx & 31);
    const int kb = (int)((idx >> 5) % KB);
    const int T = T0 + (int)((idx >> 5) / KB);
    const uint4 wv = wq[((size_t)T * KB + kb) * 32 + lane];
    const uint2 s2 = sz[((size_t)T * NG + kb / 2) * 8 + (lane >> 2)];
    const float2 sc = __half22float2(*reinterpret_cast<const __half2*>(&s2.x));
    const float zl = (float)((int)(s2.y & 0xFFFFu) - 0x4300);
    const float zh = (float)((int)(s2.y >> 16) - 0x4300);
    const uint32_t wr[4] = {wv.x, wv.y, wv.z, wv.w};
    __align__(16) __nv_bfloat16 lo[16], hi[16];
#pragma unroll
    for (int s = 0; s < 4; ++s)
#pragma unroll
      for (int i = 0; i < 8; ++i) {     // nibble i = h + 2c + 4p -> column 4s + 2c + p of row h
        const int h = i & 1, c = (i >> 1) & 1, pp = i >> 2;
        const float q = (float)((wr[s] >> (4 * i)) & 0xF);
        if (h == 0) lo[4 * s + 2 * c + pp] = __float2bfloat16_rn((q - zl) * sc.x);
        else hi[4 * s + 2 * c + pp] = __float2bfloat16_rn((q - zh) * sc.y);
      }
    const int g = lane >> 2, t = lane & 3;
    const int r0 = (T - T0) * 16 + g, k = kb * 64 + t * 16;
    if (r0 < rows) {
      uint4* o = reinterpret_cast<uint4*>(out + (size_t)r0 * K + k);
      o[0] = reinterpret_cast<const uint4*>(lo)[0];
      o[1] = reinterpret_cast<const uint4*>(lo)[1];
    }
    if (r0 + 8 < rows) {
      uint4* o = reinterpret_cast<uint4*>(out + (size_t)(r0 + 8) * K + k);
      o[0] = reinterpret_cast<const uint4*>(hi)[0];
      o[1] = reinterpret_cast<const uint4*>(hi)[1];
    }
  }
}

}  // namespace w4

// x bf16 [M <= 8, K]; wq uint8 [Np, K/2] and sz int32 [Np/16, K/128, 8, 2] in the fragment
// layout; out bf16 [M, N] (N = out.size(1)); status = the device error word of bounded waits
void w4a16_gemv(torch::Tensor x, torch::Tensor wq, torch::Tensor sz, torch::Tensor out,
                torch::Tensor status) {
  const int M = x.size(0), K = x.size(1), N = out.size(1);
  const int ntiles = (N + 15) / 16;
  TORCH_CHECK(M >= 1 && M <= w4::MAXM && out.size(0) == M, "w4a16_gemv: 1..8 rows");
  TORCH_CHECK(K % w4::G == 0 && wq.size(1) * 2 == K && wq.size(0) == ntiles * 16,
              "w4a16_gemv: weight shape");
  TORCH_CHECK(sz.scalar_type() == at::kInt && sz.numel() == (int64_t)ntiles * (K / w4::G) * 16,
              "w4a16_gemv: scales");
  TORCH_CHECK(x.stride(1) == 1 && x.stride(0) % 8 == 0 && out.stride(1) == 1 &&
                  (reinterpret_cast<uintptr_t>(x.data_ptr()) % 16) == 0 && wq.is_contiguous() &&
                  (reinterpret_cast<uintptr_t>(wq.data_ptr()) % 16) == 0 && sz.is_contiguous() &&
                  (reinterpret_cast<uintptr_t>(sz.data_ptr()) % 16) == 0,
              "w4a16_gemv: layout");
  const at::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int NG = K / w4::G;
  // row tiles per CTA: four for vocabulary-sized N (measured 179 vs 196 us on the 248320-row
  // lm_head), two below (more CTAs); RADIANCE_W4A16_TW=2|4 overrides.  K is split over a
  // cluster until about 1000 CTAs are in flight.
  static const int tw_env = [] {
    const char* v = std::getenv("RADIANCE_W4A16_TW");
    return v ? std::atoi(v) : 0;
  }();
  const int TW = tw_env == 4 ? 4 : tw_env == 2 ? 2 : (ntiles >= 4096 ? 4 : 2);
  const int ctas = (ntiles + TW - 1) / TW;
  int C = 1;
  while (C < w4::MAXC && ctas * C < 1000 && NG >= 2 * w4::WARPS * C * 2) C *= 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas, C);
  cfg.blockDim = dim3(32 * w4::WARPS);
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = 1;
  attrs[0].val.clusterDim.y = C;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  auto kern = TW == 4 ? w4::w4a16_gemv_kernel<4, 2> : w4::w4a16_gemv_kernel<2, 3>;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern,
      (const __nv_bfloat16*)x.data_ptr(), (int)x.stride(0), (const uint4*)wq.data_ptr(),
      (const uint2*)sz.data_ptr(), N, K, M, (__nv_bfloat16*)out.data_ptr(), (int)out.stride(0),
      status.data_ptr<int>()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void w4a16_dequant(torch::Tensor wq, torch::Tensor sz, int64_t n0, torch::Tensor out) {
  const int K = wq.size(1) * 2;
  const int rows = out.size(0);
  TORCH_CHECK(out.size(1) == K && out.is_contiguous() && n0 % 16 == 0 && K % w4::G == 0 &&
                  n0 + rows <= wq.size(0), "w4a16_dequant: shapes");
  const at::cuda::CUDAGuard guard(wq.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  w4::w4a16_dequant_kernel<<<1184, 256, 0, stream>>>(
      (const uint4*)wq.data_ptr(), (const uint2*)sz.data_ptr(), K, (int)n0, rows,
      (__nv_bfloat16*)out.data_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace rad
