// Two-shot tensor-parallel all-reduce over NVLink peer memory for prefill-sized messages, fused
// with the next layer's residual add + RMSNorm(1 + w) + e4m3 quantisation.
//
// Reference behaviour: the reference's custom all-reduce bands (radiance_allreduce.py:13-27:
// one-shot for a few tokens, two-shot reduce-scatter + all-gather up to 4096 tokens, RCCL above)
// and its AR + add + RMSNorm + quant fusion (radiance_arnq.py:78-127, ar_oneshot_2rank_exact_nq in
// sly/r4d/r4d_extras_rx10.patch:181-368).  Here the two-shot path covers every prefill chunk, and
// its reduce-scatter half can be issued by the row-parallel GEMM itself.
//
// Rows are owned in contiguous blocks of `per` rows (rank o owns [o * per, (o + 1) * per)).  One
// symmetric buffer per rank (IPC-mapped into every peer) holds a header, the reduce-scatter slots
// (world source slots x per rows x H bf16) and the all-gather rows (M x H bf16).  Data moves only
// by PUSH (plain 16-byte stores to peer memory), ordered by system-scope fences and flags:
//   A0  every CTA stores its share of this rank's partial rows into the owners' slots, then adds 1
//       to each owner's arrival counter of this source (skipped when the row-parallel GEMM already
//       pushed its output tiles from its epilogue: each GEMM CTA adds 1 instead);
//   A   the owner waits for every source's count, sums its rows in fp32, stores the bf16 sums into
//       every rank's all-gather rows and releases one flag per (owner, CTA) in every rank, the
//       call's sequence number as its value (the last CTA first resets the arrival counters);
//   B   every rank waits for the flags of the rows it finishes and runs the row epilogue on its
//       local all-gather rows: bf16 copy, or residual add + RMSNorm + e4m3.
// A rank reaches its next call only after every owner released all its flags of this call, so
// slots and counters are never overwritten while a peer still reads them; all waits are bounded
// (status word).  The grid stays within one wave (every CTA resident) so phase B never waits for
// a CTA of its own rank that has not started.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace rad {
namespace ts {

constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 160;
constexpr int kCntOff = 0;            // uint32 [8]: arrivals per source
constexpr int kEpochOff = 64;         // uint32: sequence of the last completed call
constexpr int kDoneAOff = 68;         // uint32: CTAs past phase A (self-resetting)
constexpr int kDoneBOff = 72;         // uint32: CTAs past phase B (self-resetting)
constexpr int kFlagOff = 256;         // uint32 [8 owners][kMaxCtas]
constexpr int kHeaderBytes = 8192;
constexpr uint64_t kPeerWaitNs = 5ull * 1000ull * 1000ull * 1000ull;
constexpr int kMaxV = 5;              // fused rows: H <= 5 * 256 * 8

struct TsArgs {
  uint8_t* peer[kMaxRanks];   // every rank's buffer (own at `rank`)
  int world, rank;
  int M, H, per;              // rows, row length, rows per owner
  int64_t ag_off;             // byte offset of the all-gather rows (after the slots)
};

DEVI uint32_t* cnt_of(uint8_t* base) { return reinterpret_cast<uint32_t*>(base + kCntOff); }
DEVI uint32_t* flag_of(uint8_t* base, int owner, int cta) {
  return reinterpret_cast<uint32_t*>(base + kFlagOff) + owner * kMaxCtas + cta;
}
DEVI __nv_bfloat16* slot_row(const TsArgs& a, int owner, int src, int local) {
  return reinterpret_cast<__nv_bfloat16*>(a.peer[owner] + kHeaderBytes) +
         ((size_t)src * a.per + local) * a.H;
}
DEVI __nv_bfloat16* ag_row(const TsArgs& a, int dest, int row) {
  return reinterpret_cast<__nv_bfloat16*>(a.peer[dest] + a.ag_off) + (size_t)row * a.H;
}
DEVI void red_add_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

template <bool FUSED, bool PUSHED>
__global__ void __launch_bounds__(256) ts_allreduce_kernel(
    const TsArgs a, const __nv_bfloat16* __restrict__ inp, unsigned expected,
    __nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ residual,
    const __nv_bfloat16* __restrict__ w, float eps, __nv_bfloat16* __restrict__ res_out,
    uint8_t* __restrict__ q, float* __restrict__ scale, int* __restrict__ status) {
  uint4 wpre[kMaxV];
  if constexpr (FUSED) {
#pragma unroll
    for (int i = 0; i < kMaxV; ++i) {
      const int v = threadIdx.x + i * 256;
      wpre[i] = v < a.H / 8 ? reinterpret_cast<const uint4*>(w)[v] : make_uint4(0, 0, 0, 0);
    }
  }
  pdl_wait();     // this rank's partial (or its GEMM's pushes) precede this kernel
  pdl_trigger();
  __shared__ bool s_last;
  __shared__ int s_ok;
  __shared__ float red[8];
  const int G = gridDim.x, c = blockIdx.x;
  const int H = a.H, nv = H / 8;
  uint8_t* mine = a.peer[a.rank];
  const uint32_t seq = *reinterpret_cast<volatile uint32_t*>(mine + kEpochOff) + 1u;
  if (threadIdx.x == 0) s_ok = 1;

  // ---- A0: push this rank's partial rows to their owners ----
  if constexpr (!PUSHED) {
    const int rpc = (a.M + G - 1) / G;
    const int r0 = c * rpc, r1 = min(a.M, r0 + rpc);
    for (int r = r0; r < r1; ++r) {
      const int o = r / a.per;
      __nv_bfloat16* dst = slot_row(a, o, a.rank, r - o * a.per);
      const uint4* src = reinterpret_cast<const uint4*>(inp + (size_t)r * H);
      for (int v = threadIdx.x; v < nv; v += 256) reinterpret_cast<uint4*>(dst)[v] = src[v];
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0)
      for (int o = 0; o < a.world; ++o) red_add_release_sys(cnt_of(a.peer[o]) + a.rank, 1u);
  }

  // ---- A: reduce my rows over every source, all-gather them ----
  const int my0 = a.rank * a.per;
  const int nmy = max(0, min(a.per, a.M - my0));
  {
    const int rpc = (nmy + G - 1) / G;
    const int l0 = c * rpc, l1 = min(nmy, l0 + rpc);
    if (threadIdx.x == 0) {
      for (int p = 0; p < a.world; ++p)
        if (!wait_flag_geq(cnt_of(mine) + p, expected, status, kErrPeerTimeout, kPeerWaitNs)) s_ok = 0;
    }
    __syncthreads();
    if (s_ok) {
      for (int l = l0; l < l1; ++l) {
        for (int v = threadIdx.x; v < nv; v += 256) {
          float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
          for (int p = 0; p < a.world; ++p) {
            const uint4 u = reinterpret_cast<const uint4*>(slot_row(a, a.rank, p, l))[v];
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float2 f = __bfloat1622float2(h[i]);
              acc[2 * i] += f.x;
              acc[2 * i + 1] += f.y;
            }
          }
          uint4 o;
          __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
          for (int i = 0; i < 4; ++i) oh[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
          for (int d = 0; d < a.world; ++d) reinterpret_cast<uint4*>(ag_row(a, d, my0 + l))[v] = o;
        }
      }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      // the last CTA past its reads resets the arrival counters before releasing its flags
      const unsigned old = atomicAdd(reinterpret_cast<uint32_t*>(mine + kDoneAOff), 1u);
      if (old == (unsigned)(G - 1)) {
        for (int p = 0; p < a.world; ++p) cnt_of(mine)[p] = 0u;
        *reinterpret_cast<uint32_t*>(mine + kDoneAOff) = 0u;
        __threadfence_system();
      }
      for (int d = 0; d < a.world; ++d) st_release_sys(flag_of(a.peer[d], a.rank, c), seq);
    }
  }

  // ---- B: the row epilogue on the local all-gather rows ----
  {
    const int rpc = (a.M + G - 1) / G;
    const int r0 = c * rpc, r1 = min(a.M, r0 + rpc);
    int waited_o = -1, waited_c = -1;
    for (int r = r0; r < r1; ++r) {
      const int o = r / a.per;
      const int n_o = max(0, min(a.per, a.M - o * a.per));
      const int oc = (r - o * a.per) / ((n_o + G - 1) / G);
      if (o != waited_o || oc != waited_c) {
        __syncthreads();
        if (threadIdx.x == 0 &&
            !wait_flag_geq(flag_of(mine, o, oc), seq, status, kErrPeerTimeout, kPeerWaitNs))
          s_ok = 0;
        __syncthreads();
        waited_o = o;
        waited_c = oc;
      }
      const __nv_bfloat16* row = ag_row(a, a.rank, r);
      if constexpr (!FUSED) {
        for (int v = threadIdx.x; v < nv; v += 256)
          reinterpret_cast<uint4*>(out + (size_t)r * H)[v] = reinterpret_cast<const uint4*>(row)[v];
      } else {
        float vals[kMaxV][8];
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < kMaxV; ++i) {
          const int v = threadIdx.x + i * 256;
          if (v < nv) {
            const uint4 su = reinterpret_cast<const uint4*>(row)[v];
            const uint4 ru = reinterpret_cast<const uint4*>(residual + (size_t)r * H)[v];
            const __nv_bfloat162* sh = reinterpret_cast<const __nv_bfloat162*>(&su);
            const __nv_bfloat162* rh = reinterpret_cast<const __nv_bfloat162*>(&ru);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float2 fs = __bfloat1622float2(sh[k]), fr = __bfloat1622float2(rh[k]);
              vals[i][2 * k] = fs.x + fr.x;
              vals[i][2 * k + 1] = fs.y + fr.y;
            }
            uint4 o;
            __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
            for (int k = 0; k < 4; ++k) oh[k] = __floats2bfloat162_rn(vals[i][2 * k], vals[i][2 * k + 1]);
            reinterpret_cast<uint4*>(res_out + (size_t)r * H)[v] = o;
#pragma unroll
            for (int j = 0; j < 8; ++j) ss += vals[i][j] * vals[i][j];
          }
        }
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();
        ss = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += red[i];
        __syncthreads();
        const float rs = rsqrtf(ss / (float)H + eps);
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < kMaxV; ++i) {
          const int v = threadIdx.x + i * 256;
          if (v < nv) {
            const __nv_bfloat162* wh = reinterpret_cast<const __nv_bfloat162*>(&wpre[i]);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float2 f = __bfloat1622float2(wh[k]);
              vals[i][2 * k] = bf16_round(vals[i][2 * k] * rs * (f.x + 1.f));
              vals[i][2 * k + 1] = bf16_round(vals[i][2 * k + 1] * rs * (f.y + 1.f));
              amax = fmaxf(amax, fmaxf(fabsf(vals[i][2 * k]), fabsf(vals[i][2 * k + 1])));
            }
          }
        }
        amax = warp_max(amax);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
        __syncthreads();
        amax = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, red[i]);
        __syncthreads();
        const float sc = fmaxf(amax / 448.f, 1.f / (448.f * 512.f));
        const float inv = 1.f / sc;
#pragma unroll
        for (int i = 0; i < kMaxV; ++i) {
          const int v = threadIdx.x + i * 256;
          if (v < nv) {
            uint2 u;
            uint16_t* hh = reinterpret_cast<uint16_t*>(&u);
#pragma unroll
            for (int k = 0; k < 4; ++k) hh[k] = f32x2_to_e4m3x2(vals[i][2 * k] * inv, vals[i][2 * k + 1] * inv);
            reinterpret_cast<uint2*>(q + (size_t)r * H)[v] = u;
          }
        }
        if (threadIdx.x == 0) scale[r] = sc;
      }
    }
  }
  // the last CTA publishes this call's sequence (the next call's flags carry seq + 1)
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned old = atomicAdd(reinterpret_cast<uint32_t*>(mine + kDoneBOff), 1u);
    if (old == (unsigned)(G - 1)) {
      *reinterpret_cast<uint32_t*>(mine + kDoneBOff) = 0u;
      *reinterpret_cast<volatile uint32_t*>(mine + kEpochOff) = seq;
    }
  }
}

}  // namespace ts

int64_t ts_header_bytes() { return ts::kHeaderBytes; }

// Buffer bytes of the two-shot all-reduce for up to mmax rows of H features (any world size):
// header + reduce-scatter slots (world x per x H bf16 <= (mmax + world * 8) x H) + gather rows.
int64_t ts_buffer_bytes(int64_t mmax, int64_t H) {
  return ts::kHeaderBytes + ((mmax + 8 * ts::kMaxRanks) * H * 2 + 255) / 256 * 256 + mmax * H * 2;
}

static int ts_grid(int M) {
  static int sms = [] {
    int dev = 0, v = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  return std::max(1, std::min({M, sms, ts::kMaxCtas}));
}

// rows per owner for M rows over `world` ranks (multiple of 8 keeps 16-byte row starts for any H)
int64_t ts_rows_per_rank(int64_t M, int64_t world) { return (M + world * 8 - 1) / (world * 8) * 8; }

// Two-shot all-reduce of x [M, H] bf16 (this rank's partial) over the ranks' buffers `peers`.
// pushed: the row-parallel GEMM already stored x into the owners' slots (x unused, expected =
// its CTA count); otherwise phase A0 pushes x.  Fused (q defined): residual add + RMSNorm(1 + w) +
// e4m3 -> res_out, q, scale; plain: out = sum.
void ts_allreduce(std::vector<int64_t> peers, int64_t rank, int64_t M, int64_t H,
                  int64_t buf_bytes, torch::Tensor x, bool pushed, int64_t expected,
                  torch::Tensor out, torch::Tensor residual, torch::Tensor weight, double eps,
                  torch::Tensor res_out, torch::Tensor q, torch::Tensor scale,
                  torch::Tensor status) {
  using namespace ts;
  const int world = peers.size();
  TORCH_CHECK(world >= 1 && world <= kMaxRanks, "ts_allreduce: world size");
  TORCH_CHECK(H % 8 == 0 && H <= kMaxV * 256 * 8, "ts_allreduce: H % 8 and H <= 10240");
  TORCH_CHECK(ts_buffer_bytes(M, H) <= buf_bytes, "ts_allreduce: message exceeds the buffer");
  if (M == 0) return;
  TsArgs a{};
  for (int i = 0; i < world; ++i) a.peer[i] = (uint8_t*)(uintptr_t)peers[i];
  a.world = world;
  a.rank = (int)rank;
  a.M = (int)M;
  a.H = (int)H;
  a.per = (int)ts_rows_per_rank(M, world);
  a.ag_off = kHeaderBytes + ((int64_t)a.per * world * H * 2 + 255) / 256 * 256;
  const bool fused = q.defined() && q.numel();
  if (!pushed) {
    TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.size(0) == M &&
                    x.size(1) == H, "ts_allreduce: x");
  }
  if (fused) {
    TORCH_CHECK(residual.is_contiguous() && res_out.is_contiguous() && q.is_contiguous() &&
                    weight.numel() >= H, "ts_allreduce: fused operands");
  } else {
    TORCH_CHECK(out.is_contiguous() && out.size(0) >= M && out.size(1) == H, "ts_allreduce: out");
  }
  const int G = ts_grid((int)M);
  const unsigned exp = pushed ? (unsigned)expected : (unsigned)G;
  const at::cuda::CUDAGuard guard(fused ? q.device() : out.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  int* st = status.numel() ? status.data_ptr<int>() : nullptr;
  const __nv_bfloat16* xp = pushed ? nullptr : (const __nv_bfloat16*)x.data_ptr();
  auto bfp = [](const torch::Tensor& t) {
    return t.defined() && t.numel() ? (__nv_bfloat16*)t.data_ptr() : nullptr;
  };
#define TS_LAUNCH(F, P)                                                                           \
  C10_CUDA_CHECK(launch_pdl((ts_allreduce_kernel<F, P>), dim3(G), dim3(256), 0, stream, a, xp,   \
                            exp, bfp(out), bfp(residual), bfp(weight), (float)eps, bfp(res_out),  \
                            fused ? (uint8_t*)q.data_ptr() : nullptr,                             \
                            fused ? scale.data_ptr<float>() : nullptr, st))
  if (fused && pushed) TS_LAUNCH(true, true);
  else if (fused) TS_LAUNCH(true, false);
  else if (pushed) TS_LAUNCH(false, true);
  else TS_LAUNCH(false, false);
#undef TS_LAUNCH
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace rad
