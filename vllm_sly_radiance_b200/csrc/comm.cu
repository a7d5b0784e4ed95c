// Tensor-parallel collectives over NVLink / NVSwitch peer memory.
//
// Reference behaviour: RadianceAllreduce (radiance_allreduce.py:65-358) and libr4d
// ar_oneshot_* / ar_twoshot_* / ar_oneshot_2rank_exact_nq (sly/r4d/r4d_extras_rx10.patch:181-368):
// push all-reduce over P2P IPC scratch with per-block flag + sequence handshake, optionally fused
// with the next layer's residual add + Gemma RMSNorm + e4m3 quant ("fp8 residual-stream contract").
//
// B200 design:
//  * Each rank owns one symmetric buffer (cudaMalloc'd, IPC-mapped into every peer).  Data moves
//    by PUSH: a rank stores its rows into its own source slot of every peer's buffer, and each
//    rank reduces only its local slots, so nothing is ever read across NVLink.
//  * Flag-in-word ("LL") stores: every 8-byte word carries 4 bytes of payload (two bf16) and the
//    32-bit sequence number of the call that wrote it.  The reader polls each word until its
//    sequence matches, so no system-scope fence, flag or counter sits between data and reader:
//    an 8-byte store is seen whole.  Sequence numbers live in device memory (per-CTA counter for
//    the one-shot, per-buffer epoch for the GEMM push), so the kernels replay inside CUDA graphs.
//    Two parity halves keep a fast rank from overwriting words a slow peer has not read yet.
//    Every poll is bounded: on timeout the CTA records kErrPeerTimeout and returns.
//  * One-shot all-reduce: CTA c pushes rows [c*rows, ...) to every peer, then reduces the same
//    rows from the `world` local source slots in fp32.  Fused variant: each reduced row goes
//    through residual add + RMSNorm(1+w) + per-row e4m3 quant (the producer of the next linear).
//  * GEMM push: the row-parallel GEMM's epilogue writes its tile as LL words straight into every
//    peer (mxfp4_gemm.cu); push_recv_kernel is the reducing half.
//  * Plain loads and stores to peer memory only; no bulk-copy engine touches a peer address.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <map>
#include <mutex>
#include <string>

#include <vector>

#include "common.cuh"

namespace rad {
namespace comm {

constexpr int kMaxRanks = 8;
constexpr uint64_t kPeerWaitNs = 5ull * 1000ull * 1000ull * 1000ull;   // 5 s per wait
constexpr int kMaxBlocks = 64;
constexpr int kDataOffset = 256;                 // after the per-CTA sequence counters

struct PeerPtrs {
  uint8_t* p[kMaxRanks];
};

DEVI uint32_t* counters_of(uint8_t* base) { return reinterpret_cast<uint32_t*>(base); }

// poll 4 LL words (8 bf16, 32 bytes, 16-byte aligned) until all carry `seq`
DEVI bool ld_ll8(const uint64_t* p, uint32_t seq, float (&f)[8], int* status) {
  uint32_t a0, f0, a1, f1, a2, f2, a3, f3;
  uint64_t t0 = 0;
  const uint64_t limit = wait_limit_ns(status, 3, kPeerWaitNs);
  for (int it = 0;; ++it) {
    asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(a0), "=r"(f0), "=r"(a1), "=r"(f1) : "l"(p) : "memory");
    asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(a2), "=r"(f2), "=r"(a3), "=r"(f3) : "l"(p + 2) : "memory");
    if (f0 == seq && f1 == seq && f2 == seq && f3 == seq) break;
    if ((it & 63) == 0) {
      const uint64_t now = globaltimer_ns();
      if (it == 0) t0 = now;
      else if (now - t0 > limit) {
        if (status) atomicExch(status, kErrPeerTimeout);
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = 0.f;
        return false;
      }
    }
  }
  const uint32_t w[4] = {a0, a1, a2, a3};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
    const float2 v = __bfloat1622float2(h);
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
  return true;
}

// store 8 bf16 (one uint4) as 4 LL words
DEVI void st_ll8(uint64_t* p, uint4 u, uint32_t seq) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(u.x), "r"(seq),
               "r"(u.y), "r"(seq) : "memory");
  asm volatile("st.volatile.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p + 2), "r"(u.z), "r"(seq),
               "r"(u.w), "r"(seq) : "memory");
}

// Sum rows [r0, r1) over `world` LL sources (row r of source p at srcs[p] + r * H / 2 words) in
// fp32; plain: write the bf16 sum to out; fused: s = bf16(sum) + residual -> res_out, Gemma
// RMSNorm (1 + w), per-row e4m3 quant.  False if a wait timed out.
constexpr int kFusedMaxV = 5;   // fused rows: H <= 5 * 256 * 8 = 10240

// the fused path's RMSNorm weight (a model constant), fetched by each kernel before its
// programmatic-dependency wait so the load overlaps the predecessor's tail
DEVI void prefetch_norm_weight(const __nv_bfloat16* __restrict__ w, int H, uint4 (&wpre)[kFusedMaxV]) {
#pragma unroll
  for (int i = 0; i < kFusedMaxV; ++i) {
    const int v = threadIdx.x + i * 256;
    wpre[i] = (w != nullptr && v < H / 8) ? reinterpret_cast<const uint4*>(w)[v]
                                          : make_uint4(0, 0, 0, 0);
  }
}

template <bool FUSED>
DEVI bool reduce_rows(const uint64_t* const* srcs, int world, uint32_t seq, int r0, int r1, int H,
                      __nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ residual,
                      const uint4 (&wpre)[kFusedMaxV], float eps,
                      __nv_bfloat16* __restrict__ res_out, uint8_t* __restrict__ q,
                      float* __restrict__ scale, float* red, int* status) {
  const int nv = H / 8;
  bool ok = true;
  for (int r = r0; r < r1; ++r) {
    if constexpr (!FUSED) {
      for (int v = threadIdx.x; v < nv; v += blockDim.x) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int p = 0; p < world; ++p) {
          float f[8];
          ok &= ld_ll8(srcs[p] + (size_t)r * (H / 2) + v * 4, seq, f, status);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] += f[i];
        }
        uint4 o;
        __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
        for (int i = 0; i < 4; ++i) oh[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
        reinterpret_cast<uint4*>(out + (size_t)r * H)[v] = o;
      }
    } else {
      constexpr int MAXV = kFusedMaxV;
      float vals[MAXV][8];
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        const int v = threadIdx.x + i * 256;
        if (v < nv) {
#pragma unroll
          for (int j = 0; j < 8; ++j) vals[i][j] = 0.f;
          for (int p = 0; p < world; ++p) {
            float f[8];
            ok &= ld_ll8(srcs[p] + (size_t)r * (H / 2) + v * 4, seq, f, status);
#pragma unroll
            for (int j = 0; j < 8; ++j) vals[i][j] += f[j];
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
          const __nv_bfloat162* wh = reinterpret_cast<const __nv_bfloat162*>(&wpre[i]);
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
  return ok;
}

// One-shot push all-reduce.  Buffer of each rank: [per-CTA sequence counters][data @ 256: two
// parity halves of `half_bytes`, each world source slots x M rows x H / 2 LL words].
template <bool FUSED>
__global__ void __launch_bounds__(256) oneshot_kernel(
    PeerPtrs peers, int world, int rank, const __nv_bfloat16* __restrict__ inp, int M, int H,
    int64_t half_bytes, __nv_bfloat16* __restrict__ out,
    const __nv_bfloat16* __restrict__ residual, const __nv_bfloat16* __restrict__ w, float eps,
    __nv_bfloat16* __restrict__ res_out, uint8_t* __restrict__ q, float* __restrict__ scale,
    int* __restrict__ status) {
  uint4 wpre[kFusedMaxV];
  if constexpr (FUSED) prefetch_norm_weight(w, H, wpre);
  pdl_wait();     // inputs come from the preceding kernel
  pdl_trigger();
  __shared__ uint32_t s_seq;
  __shared__ float red[8];
  const int cta = blockIdx.x;
  const int rows_per = (M + gridDim.x - 1) / gridDim.x;
  const int r0 = cta * rows_per;
  const int r1 = min(M, r0 + rows_per);
  uint8_t* mine = peers.p[rank];
  if (threadIdx.x == 0) {
    uint32_t* ctr = counters_of(mine) + cta;
    s_seq = *ctr + 1;
    *ctr = s_seq;
  }
  __syncthreads();
  const uint32_t seq = s_seq;
  const int64_t half = (int64_t)(seq & 1) * half_bytes;
  const size_t row_words = (size_t)H / 2;
  // 1) push own rows into this rank's source slot of every peer
  const int nv = H / 8;
  for (int r = r0; r < r1; ++r)
    for (int v = threadIdx.x; v < nv; v += blockDim.x) {
      const uint4 u = reinterpret_cast<const uint4*>(inp + (size_t)r * H)[v];
      for (int p = 0; p < world; ++p) {
        uint64_t* dst = reinterpret_cast<uint64_t*>(peers.p[p] + kDataOffset + half) +
                        ((size_t)rank * M + r) * row_words + v * 4;
        st_ll8(dst, u, seq);
      }
    }
  // 2) reduce the local source slots
  const uint64_t* srcs[kMaxRanks];
  for (int p = 0; p < world; ++p)
    srcs[p] = reinterpret_cast<const uint64_t*>(mine + kDataOffset + half) + (size_t)p * M * row_words;
  reduce_rows<FUSED>(srcs, world, seq, r0, r1, H, out, residual, wpre, eps, res_out, q, scale,
                     red, status);
}

// Reducing half of the GEMM-fused all-reduce: every rank's row-parallel GEMM has pushed its tile
// rows as LL words into this rank's buffer (PushArgs layout).  The last CTA to finish advances
// the epoch, which is the sequence source of the next GEMM push on this rank.
template <bool FUSED>
__global__ void __launch_bounds__(256) push_recv_kernel(
    const PushArgs pa, int M, int H, __nv_bfloat16* __restrict__ out,
    const __nv_bfloat16* __restrict__ residual, const __nv_bfloat16* __restrict__ w, float eps,
    __nv_bfloat16* __restrict__ res_out, uint8_t* __restrict__ q, float* __restrict__ scale,
    int* __restrict__ status) {
  uint4 wpre[kFusedMaxV];
  if constexpr (FUSED) prefetch_norm_weight(w, H, wpre);
  pdl_wait();     // the pushing GEMM precedes this kernel on every rank
  pdl_trigger();
  __shared__ float red[8];
  __shared__ bool s_last;
  const uint32_t seq = push_seq(pa);
  const int rows_per = (M + gridDim.x - 1) / gridDim.x;
  const int r0 = blockIdx.x * rows_per;
  const int r1 = min(M, r0 + rows_per);
  const uint64_t* srcs[kMaxRanks];
  for (int p = 0; p < pa.world; ++p) srcs[p] = push_slot(pa, pa.rank, seq & 1u, p, M);
  reduce_rows<FUSED>(srcs, pa.world, seq, r0, r1, H, out, residual, wpre, eps, res_out, q, scale,
                     red, status);
  __syncthreads();
  uint8_t* mine = pa.peer[pa.rank];
  if (threadIdx.x == 0)
    s_last = atomicAdd(reinterpret_cast<uint32_t*>(mine + kPushDoneOff), 1u) == gridDim.x - 1;
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    *reinterpret_cast<uint32_t*>(mine + kPushDoneOff) = 0u;
    *reinterpret_cast<volatile uint32_t*>(mine + kPushEpochOff) = seq;
  }
}

}  // namespace comm

// ---- IPC plumbing ----
// A tensor from the caching allocator usually sits inside a larger cudaMalloc segment, and an IPC
// handle always names the whole segment: the exported record therefore carries the tensor's
// offset inside it (found with cuMemGetAddressRange), and the opening side adds that offset to
// the mapped base.  A segment mapped twice (two buffers in one segment) is opened once and
// reference-counted.
namespace {
using GetRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
GetRangeFn get_range_fn() {
  static GetRangeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p,
                "cuMemGetAddressRange unavailable");
    return reinterpret_cast<GetRangeFn>(p);
  }();
  return fn;
}
struct Mapped {
  void* base;
  int refs;
};
std::mutex g_ipc_mu;
std::map<std::string, Mapped> g_ipc_by_handle;      // handle bytes -> mapping
std::map<int64_t, std::string> g_ipc_by_ptr;        // returned pointer -> handle bytes
}  // namespace

torch::Tensor ipc_handle(torch::Tensor buf) {
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, buf.data_ptr()));
  CUdeviceptr base = 0;
  size_t size = 0;
  TORCH_CHECK(get_range_fn()(&base, &size, (CUdeviceptr)buf.data_ptr()) == CUDA_SUCCESS,
              "ipc_handle: cuMemGetAddressRange failed");
  const int64_t off = (int64_t)((uintptr_t)buf.data_ptr() - (uintptr_t)base);
  auto out = torch::empty({(int64_t)(sizeof(h) + sizeof(off))}, torch::kUInt8);
  memcpy(out.data_ptr(), &h, sizeof(h));
  memcpy((uint8_t*)out.data_ptr() + sizeof(h), &off, sizeof(off));
  return out;
}

int64_t ipc_open(torch::Tensor handle) {
  cudaIpcMemHandle_t h;
  TORCH_CHECK(handle.numel() == (int64_t)(sizeof(h) + sizeof(int64_t)), "ipc_open: record size");
  memcpy(&h, handle.data_ptr(), sizeof(h));
  int64_t off = 0;
  memcpy(&off, (const uint8_t*)handle.data_ptr() + sizeof(h), sizeof(off));
  const std::string key(reinterpret_cast<const char*>(&h), sizeof(h));
  std::lock_guard<std::mutex> lk(g_ipc_mu);
  auto it = g_ipc_by_handle.find(key);
  void* base = nullptr;
  if (it == g_ipc_by_handle.end()) {
    C10_CUDA_CHECK(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
    g_ipc_by_handle[key] = Mapped{base, 1};
  } else {
    base = it->second.base;
    it->second.refs += 1;
  }
  const int64_t ptr = (int64_t)((uintptr_t)base + off);
  g_ipc_by_ptr[ptr] = key;
  return ptr;
}

void ipc_close(int64_t ptr) {
  std::lock_guard<std::mutex> lk(g_ipc_mu);
  auto pit = g_ipc_by_ptr.find(ptr);
  TORCH_CHECK(pit != g_ipc_by_ptr.end(), "ipc_close: pointer was not opened here");
  auto it = g_ipc_by_handle.find(pit->second);
  g_ipc_by_ptr.erase(pit);
  if (it != g_ipc_by_handle.end() && --it->second.refs == 0) {
    C10_CUDA_CHECK(cudaIpcCloseMemHandle(it->second.base));
    g_ipc_by_handle.erase(it);
  }
}

int64_t symm_header_bytes() { return comm::kDataOffset; }

// peers: int64 device pointers of every rank's symmetric buffer (own included at `rank`);
// half_bytes: capacity of one parity half of the data region
void allreduce_oneshot(std::vector<int64_t> peers, int64_t rank, torch::Tensor inp,
                       int64_t half_bytes, torch::Tensor out, torch::Tensor residual,
                       torch::Tensor weight, double eps, torch::Tensor res_out, torch::Tensor q,
                       torch::Tensor scale, int64_t num_blocks, torch::Tensor status) {
  using namespace comm;
  const int world = peers.size();
  TORCH_CHECK(world >= 1 && world <= kMaxRanks, "world size");
  const int M = inp.size(0), H = inp.size(1);
  TORCH_CHECK(H % 8 == 0 && H <= 10240, "allreduce: H % 8 and H <= 10240");
  TORCH_CHECK((int64_t)world * M * H * 4 <= half_bytes, "allreduce: message exceeds the symmetric buffer");
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
        pp, world, rank, (const __nv_bfloat16*)inp.data_ptr(), M, H, half_bytes, nullptr,
        (const __nv_bfloat16*)residual.data_ptr(), (const __nv_bfloat16*)weight.data_ptr(),
        (float)eps, (__nv_bfloat16*)res_out.data_ptr(), (uint8_t*)q.data_ptr(),
        scale.data_ptr<float>(), st));
  else
C10_CUDA_CHECK(launch_pdl((oneshot_kernel<false>), dim3(nb), dim3(256), 0, stream, 
        pp, world, rank, (const __nv_bfloat16*)inp.data_ptr(), M, H, half_bytes,
        (__nv_bfloat16*)out.data_ptr(), nullptr, nullptr, 0.f, nullptr, nullptr, nullptr, st));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int64_t push_buffer_bytes(int64_t world, int64_t mmax, int64_t H) {
  // header + two parity halves of world x mmax x H/2 LL words (8 bytes)
  return kPushDataOff + 2 * world * mmax * (H / 2) * 8;
}

// peers: every rank's push receive buffer (own at `rank`); half_words = words per parity half
void push_allreduce_recv(std::vector<int64_t> peers, int64_t rank, int64_t M, int64_t H,
                         int64_t half_words, torch::Tensor out, torch::Tensor residual,
                         torch::Tensor weight, double eps, torch::Tensor res_out, torch::Tensor q,
                         torch::Tensor scale, int64_t num_blocks, torch::Tensor status) {
  using namespace comm;
  const int world = peers.size();
  TORCH_CHECK(world >= 1 && world <= kMaxRanks, "world size");
  TORCH_CHECK(H % 8 == 0 && H <= 10240, "push recv: H % 8 and H <= 10240");
  TORCH_CHECK((int64_t)world * M * (H / 2) <= half_words, "push recv: message exceeds the buffer");
  if (M == 0) return;
  PushArgs pa{};
  for (int i = 0; i < world; ++i) pa.peer[i] = (uint8_t*)(uintptr_t)peers[i];
  pa.world = world;
  pa.rank = (int)rank;
  pa.half_words = half_words;
  pa.ld = (int)H;
  int nb = (int)std::min<int64_t>(num_blocks > 0 ? num_blocks : M, kMaxBlocks);
  nb = std::max(1, std::min<int>(nb, (int)M));
  const at::cuda::CUDAGuard guard(out.defined() && out.numel() ? out.device() : res_out.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  int* st = status.numel() ? status.data_ptr<int>() : nullptr;
  const bool fused = q.defined() && q.numel();
  if (fused)
    C10_CUDA_CHECK(launch_pdl((push_recv_kernel<true>), dim3(nb), dim3(256), 0, stream, pa, (int)M,
        (int)H, nullptr, (const __nv_bfloat16*)residual.data_ptr(),
        (const __nv_bfloat16*)weight.data_ptr(), (float)eps, (__nv_bfloat16*)res_out.data_ptr(),
        (uint8_t*)q.data_ptr(), scale.data_ptr<float>(), st));
  else
    C10_CUDA_CHECK(launch_pdl((push_recv_kernel<false>), dim3(nb), dim3(256), 0, stream, pa, (int)M,
        (int)H, (__nv_bfloat16*)out.data_ptr(), nullptr, nullptr, 0.f, nullptr, nullptr, nullptr,
        st));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace rad
