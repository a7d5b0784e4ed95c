// Tensor-parallel collectives over NVLink / NVSwitch peer memory.
//
// Reference behaviour: RadianceAllreduce (radiance_allreduce.py:65-358) and libr4d
// ar_oneshot_* / ar_twoshot_* / ar_oneshot_2rank_exact_nq (sly/r4d/r4d_extras_rx10.patch:181-368):
// push all-reduce over P2P IPC scratch with per-block flag + sequence handshake, optionally fused
// with the next layer's residual add + Gemma RMSNorm + e4m3 quant ("fp8 residual-stream contract").
//
// B200 design:
//  * Each rank owns one symmetric buffer (cudaMalloc'd, IPC-mapped into every peer).  Layout:
//    [flags: kMaxBlocks x kMaxRanks u32][counters: kMaxBlocks u32][data: 2 parity slots].
//  * One-shot all-reduce, per CTA: copy own row chunk into the parity slot, release-store the
//    sequence number into every peer's flag[cta][me], acquire-poll own flag[cta][p] for all p
//    (bounded: after the timeout the CTA records kErrPeerTimeout in the status word and returns),
//    then read the chunk from all peers' slots and reduce in fp32.  Sequence numbers live in
//    device memory (per-CTA counter), so the kernel replays inside CUDA graphs.  Parity double
//    buffering keeps a fast rank from overwriting a slot a slow peer still reads.
//  * Fused epilogue variant: rows are owned whole by one CTA, so the reduced row goes straight
//    through residual add + RMSNorm(1+w) + per-row e4m3 quant (the producer of the next linear).
//  * Plain loads and stores to peer memory only; no bulk-copy engine touches a peer address.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

#include "common.cuh"

namespace rad {
namespace comm {

constexpr int kMaxRanks = 8;
constexpr uint64_t kPeerWaitNs = 5ull * 1000ull * 1000ull * 1000ull;   // 5 s per handshake
constexpr int kMaxBlocks = 64;
constexpr int kHeaderBytes = kMaxBlocks * kMaxRanks * 4 + kMaxBlocks * 4;
constexpr int kDataOffset = (kHeaderBytes + 255) / 256 * 256;

struct PeerPtrs {
  uint8_t* p[kMaxRanks];
};

DEVI uint32_t* flags_of(uint8_t* base) { return reinterpret_cast<uint32_t*>(base); }
DEVI uint32_t* counters_of(uint8_t* base) {
  return reinterpret_cast<uint32_t*>(base + kMaxBlocks * kMaxRanks * 4);
}

// rows [M, H] bf16; each CTA owns a contiguous set of rows.  Output either bf16 sum or the fused
// add + RMSNorm + quant triple.
template <bool FUSED>
__global__ void __launch_bounds__(256) oneshot_kernel(
    PeerPtrs peers, int world, int rank, const __nv_bfloat16* __restrict__ inp, int M, int H,
    int64_t slot_bytes, __nv_bfloat16* __restrict__ out,
    const __nv_bfloat16* __restrict__ residual, const __nv_bfloat16* __restrict__ w, float eps,
    __nv_bfloat16* __restrict__ res_out, uint8_t* __restrict__ q, float* __restrict__ scale,
    int* __restrict__ status) {
  pdl_wait();     // inputs come from the preceding kernel
  pdl_trigger();
  __shared__ uint32_t s_seq;
  __shared__ float red[8];
  __shared__ int s_ok;
  const int cta = blockIdx.x;
  const int rows_per = (M + gridDim.x - 1) / gridDim.x;
  const int r0 = cta * rows_per;
  const int r1 = min(M, r0 + rows_per);
  uint8_t* mine = peers.p[rank];
  if (threadIdx.x == 0) {
    uint32_t* ctr = counters_of(mine) + cta;
    s_seq = *ctr + 1;
    *ctr = s_seq;
    s_ok = 1;
  }
  __syncthreads();
  const uint32_t seq = s_seq;
  const int par = seq & 1;
  // 1) own rows -> own parity slot
  __nv_bfloat16* my_slot = reinterpret_cast<__nv_bfloat16*>(mine + kDataOffset + par * slot_bytes);
  const int nv = H / 8;
  for (int r = r0; r < r1; ++r)
    for (int v = threadIdx.x; v < nv; v += blockDim.x)
      reinterpret_cast<uint4*>(my_slot + (size_t)r * H)[v] = reinterpret_cast<const uint4*>(inp + (size_t)r * H)[v];
  __threadfence_system();
  __syncthreads();
  // 2) signal every peer, 3) wait for every peer
  if (threadIdx.x < world) {
    const int p = threadIdx.x;
    st_release_sys(flags_of(peers.p[p]) + cta * kMaxRanks + rank, seq);
  }
  if (threadIdx.x < world) {
    const int p = threadIdx.x;
    if (!wait_flag_geq(flags_of(mine) + cta * kMaxRanks + p, seq, status, kErrPeerTimeout,
                        kPeerWaitNs))
      atomicExch(&s_ok, 0);
  }
  __syncthreads();
  if (!s_ok) return;
  // 4) reduce
  for (int r = r0; r < r1; ++r) {
    if constexpr (!FUSED) {
      for (int v = threadIdx.x; v < nv; v += blockDim.x) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int p = 0; p < world; ++p) {
          const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(peers.p[p] + kDataOffset + par * slot_bytes);
          uint4 u = reinterpret_cast<const uint4*>(src + (size_t)r * H)[v];
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float2 f = __bfloat1622float2(h[i]);
            acc[2 * i] += f.x;
            acc[2 * i + 1] += f.y;
          }
        }
        uint4 o;
        __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
        for (int i = 0; i < 4; ++i) oh[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
        reinterpret_cast<uint4*>(out + (size_t)r * H)[v] = o;
      }
    } else {
      // fused: s = bf16(sum) + residual (fp32), res_out = bf16(s), n = bf16(s*rs*(1+w)), quant
      constexpr int MAXV = 5;   // H <= 5 * 256 * 8 = 10240
      float vals[MAXV][8];
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        const int v = threadIdx.x + i * 256;
        if (v < nv) {
#pragma unroll
          for (int j = 0; j < 8; ++j) vals[i][j] = 0.f;
          for (int p = 0; p < world; ++p) {
            const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(peers.p[p] + kDataOffset + par * slot_bytes);
            uint4 u = reinterpret_cast<const uint4*>(src + (size_t)r * H)[v];
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              float2 f = __bfloat1622float2(h[k]);
              vals[i][2 * k] += f.x;
              vals[i][2 * k + 1] += f.y;
            }
          }
          uint4 ru = reinterpret_cast<const uint4*>(residual + (size_t)r * H)[v];
          const __nv_bfloat162* rh = reinterpret_cast<const __nv_bfloat162*>(&ru);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            float2 f = __bfloat1622float2(rh[k]);
            vals[i][2 * k] = bf16_round(vals[i][2 * k]) + f.x;
            vals[i][2 * k + 1] = bf16_round(vals[i][2 * k + 1]) + f.y;
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
      for (int i = 0; i < MAXV; ++i) {
        const int v = threadIdx.x + i * 256;
        if (v < nv) {
          uint4 wu = reinterpret_cast<const uint4*>(w)[v];
          const __nv_bfloat162* wh = reinterpret_cast<const __nv_bfloat162*>(&wu);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            float2 f = __bfloat1622float2(wh[k]);
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
      for (int i = 0; i < MAXV; ++i) {
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

}  // namespace comm

// ---- IPC plumbing ----
torch::Tensor ipc_handle(torch::Tensor buf) {
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, buf.data_ptr()));
  auto out = torch::empty({(int64_t)sizeof(h)}, torch::kUInt8);
  memcpy(out.data_ptr(), &h, sizeof(h));
  return out;
}

int64_t ipc_open(torch::Tensor handle) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle.data_ptr(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return (int64_t)(uintptr_t)p;
}

void ipc_close(int64_t ptr) { C10_CUDA_CHECK(cudaIpcCloseMemHandle((void*)(uintptr_t)ptr)); }

int64_t symm_header_bytes() { return comm::kDataOffset; }

// peers: int64 device pointers of every rank's symmetric buffer (own included at `rank`)
void allreduce_oneshot(std::vector<int64_t> peers, int64_t rank, torch::Tensor inp,
                       int64_t slot_bytes, torch::Tensor out, torch::Tensor residual,
                       torch::Tensor weight, double eps, torch::Tensor res_out, torch::Tensor q,
                       torch::Tensor scale, int64_t num_blocks, torch::Tensor status) {
  using namespace comm;
  const int world = peers.size();
  TORCH_CHECK(world >= 1 && world <= kMaxRanks, "world size");
  const int M = inp.size(0), H = inp.size(1);
  TORCH_CHECK(H % 8 == 0 && H <= 10240, "allreduce: H % 8 and H <= 10240");
  TORCH_CHECK((int64_t)M * H * 2 <= slot_bytes, "allreduce: message exceeds the symmetric slot");
  if (M == 0) return;
  PeerPtrs pp;
  for (int i = 0; i < kMaxRanks; ++i) pp.p[i] = i < world ? (uint8_t*)(uintptr_t)peers[i] : nullptr;
  int nb = (int)std::min<int64_t>(num_blocks > 0 ? num_blocks : M, kMaxBlocks);
  nb = std::max(1, std::min(nb, M));
  const at::cuda::CUDAGuard guard(inp.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  int* st = status.numel() ? status.data_ptr<int>() : nullptr;
  const bool fused = q.defined() && q.numel();
  if (fused)
C10_CUDA_CHECK(launch_pdl((oneshot_kernel<true>), dim3(nb), dim3(256), 0, stream, 
        pp, world, rank, (const __nv_bfloat16*)inp.data_ptr(), M, H, slot_bytes, nullptr,
        (const __nv_bfloat16*)residual.data_ptr(), (const __nv_bfloat16*)weight.data_ptr(),
        (float)eps, (__nv_bfloat16*)res_out.data_ptr(), (uint8_t*)q.data_ptr(),
        scale.data_ptr<float>(), st));
  else
C10_CUDA_CHECK(launch_pdl((oneshot_kernel<false>), dim3(nb), dim3(256), 0, stream, 
        pp, world, rank, (const __nv_bfloat16*)inp.data_ptr(), M, H, slot_bytes,
        (__nv_bfloat16*)out.data_ptr(), nullptr, nullptr, 0.f, nullptr, nullptr, nullptr, st));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace rad
