// Expert-parallel MoE dispatch / combine over NVLink peer memory (data-parallel attention: each
// rank has its own tokens, owns E / world experts).
//
// Reference behaviour: the north star's fused expert all-to-all; the reference itself serves MoE
// TP-sharded through vLLM fused_moe.  Protocol per MoE call, all on the caller's stream:
//   1. ep_dispatch: every CTA ranks the (token, k) pairs by expert (warp match, identical in
//      every CTA) and writes its share of rows straight into the owner's receive buffer in the
//      grouped GEMM's input layout: source segment [src][maxr] rows, rows of one expert
//      contiguous; e4m3 row, fp32 scale, meta = t * K + k.  The last CTA publishes the
//      per-expert counts to each owner and releases its done flag (the call's sequence number).
//   2. ep_items: the owner waits (bounded) for every source, and turns the counts into the
//      grouped GEMM work table (expert, first row, rows) over the receive buffer in place.
//   3. the grouped W4A8 GEMMs (gate_up, then down) read the receive buffer directly; between
//      them SiLU*mul + e4m3 runs on the rows the work table covers (silu_items_kernel).
//   4. ep_combine (send): each expert output row goes back into its source's combine buffer at
//      slot t * K + k; the last CTA releases the combine flag at every source.
//   5. ep_combine (reduce): the source waits for every owner, sums the K slots of each token
//      with the routing weights, and its last CTA advances the sequence number.
// Ordering between calls follows from the protocol: a rank can only start call n + 1's dispatch
// after it has every owner's call-n combine rows, which those owners send after their GEMMs
// have consumed their call-n receive buffers.  Every wait is bounded and reports through the
// status word; every index read from peer-written memory is checked before it addresses memory.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

#include "common.cuh"

namespace rad {
namespace ep {

constexpr int kMaxWorld = 8;
constexpr int kMaxExperts = 256;      // routed experts in total
constexpr int kEpochOff = 0;
constexpr int kArriveDispOff = 64;
constexpr int kArriveCombOff = 68;
constexpr int kArriveRedOff = 72;
constexpr int kDispDoneOff = 256;     // u32 [world], written by sources
constexpr int kCombDoneOff = 320;     // u32 [world], written by owners
constexpr int kNRowsOff = 384;        // int [world], local (rows received per source)
constexpr int kCountsOff = 1024;      // int [world][El], written by sources
constexpr int64_t kDataOff = 16384;

struct Args {
  uint8_t* peer[kMaxWorld];
  int world, rank;
  int maxr;            // rows per source segment
  int maxt;            // tokens per rank per call (combine buffer rows / K)
  int H, K, El;
  int64_t q_off, s_off, m_off, c_off;   // receive rows / scales / meta, combine buffer
};

DEVI uint32_t seq_of(const Args& a) {
  return *reinterpret_cast<volatile const uint32_t*>(a.peer[a.rank] + kEpochOff) + 1u;
}

// ---- 1. dispatch ----------------------------------------------------------------------------
// smem: ids[P], rank_in_expert[P], count[E], start[E]
__global__ void __launch_bounds__(512) dispatch_kernel(const __grid_constant__ Args a,
                                                       const uint8_t* __restrict__ q, int ldq,
                                                       const float* __restrict__ s,
                                                       const int* __restrict__ ids, int T,
                                                       int* __restrict__ status) {
  extern __shared__ int sm[];
  const int P = T * a.K, E = a.El * a.world;
  int* s_ids = sm;
  int* s_rank = s_ids + P;
  int* s_cnt = s_rank + P;
  int* s_start = s_cnt + E;
  __shared__ int last;
  pdl_wait();
  pdl_trigger();
  const uint32_t e = seq_of(a);
  for (int i = threadIdx.x; i < E; i += blockDim.x) s_cnt[i] = 0;
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    const int x = ids[i];
    const bool okx = x >= 0 && x < E;
    s_ids[i] = okx ? x : 0;
    if (!okx) atomicExch(status, (int)kErrBounds);
  }
  __syncthreads();
  // stable rank of every pair among the pairs of its expert (identical in every CTA)
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    for (int c = 0; c < P; c += 32) {
      const int p = c + lane;
      const int x = p < P ? s_ids[p] : -1 - lane;
      const unsigned m = __match_any_sync(0xffffffffu, x);
      const int r = __popc(m & ((1u << lane) - 1u));
      const int base = p < P ? s_cnt[x] : 0;
      __syncwarp();
      if (p < P) {
        s_rank[p] = base + r;
        if (r == 0) s_cnt[x] = base + __popc(m);
      }
      __syncwarp();
    }
  }
  __syncthreads();
  // rows of one expert are contiguous inside each destination segment
  if (threadIdx.x < a.world) {
    const int d = threadIdx.x;
    int acc = 0;
    for (int l = 0; l < a.El; ++l) {
      s_start[d * a.El + l] = acc;
      acc += s_cnt[d * a.El + l];
    }
  }
  __syncthreads();
  // this CTA's share of rows: one warp per row, 16-byte stores into the owner's buffer
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int p = blockIdx.x * nw + warp; p < P; p += gridDim.x * nw) {
    const int x = s_ids[p], d = x / a.El;
    const int slot = s_start[x] + s_rank[p];
    if (slot >= a.maxr) {
      if (lane == 0) atomicExch(status, (int)kErrBounds);
      continue;
    }
    const int t = p / a.K;
    const int64_t row = (int64_t)a.rank * a.maxr + slot;
    uint8_t* base = a.peer[d];
    const uint4* src = reinterpret_cast<const uint4*>(q + (size_t)t * ldq);
    uint4* dst = reinterpret_cast<uint4*>(base + a.q_off + row * a.H);
    for (int c = lane; c < a.H / 16; c += 32) dst[c] = src[c];
    if (lane == 0) {
      reinterpret_cast<float*>(base + a.s_off)[row] = s[t];
      reinterpret_cast<int*>(base + a.m_off)[row] = p;      // t * K + k
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* arrive = reinterpret_cast<uint32_t*>(a.peer[a.rank] + kArriveDispOff);
    last = atomicAdd(arrive, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence_system();
  // counts of this source's rows per expert, then the done flag, at every owner
  for (int i = threadIdx.x; i < E; i += blockDim.x) {
    const int d = i / a.El, l = i % a.El;
    reinterpret_cast<volatile int*>(a.peer[d] + kCountsOff)[a.rank * a.El + l] = s_cnt[i];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < a.world)
    st_release_sys(reinterpret_cast<uint32_t*>(a.peer[threadIdx.x] + kDispDoneOff) + a.rank, e);
  if (threadIdx.x == 0) *reinterpret_cast<uint32_t*>(a.peer[a.rank] + kArriveDispOff) = 0;
}

// ---- 2. work table -----------------------------------------------------------------------------
// items int32 [max_items][3] = (local expert, first row, rows), rows = 0 past the end
__global__ void items_kernel(const __grid_constant__ Args a, int bn, int* __restrict__ items,
                             int max_items, int* __restrict__ status) {
  __shared__ int s_cnt[kMaxExperts];   // [src][El]
  __shared__ int s_off[kMaxExperts];   // row offset of (src, expert) inside the src segment
  __shared__ int s_n;
  pdl_wait();
  pdl_trigger();
  const uint32_t e = seq_of(a);
  const uint8_t* me = a.peer[a.rank];
  if (threadIdx.x < a.world)
    wait_flag_geq(reinterpret_cast<const uint32_t*>(me + kDispDoneOff) + threadIdx.x, e, status,
                  kErrPeerTimeout);
  __syncthreads();
  for (int i = threadIdx.x; i < a.world * a.El; i += blockDim.x)
    s_cnt[i] = reinterpret_cast<volatile const int*>(me + kCountsOff)[i];
  __syncthreads();
  if (threadIdx.x < a.world) {
    int acc = 0;
    for (int l = 0; l < a.El; ++l) {
      s_off[threadIdx.x * a.El + l] = acc;
      acc += s_cnt[threadIdx.x * a.El + l];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int n = 0;
    for (int l = 0; l < a.El; ++l)
      for (int src = 0; src < a.world; ++src) {
        const int off = s_off[src * a.El + l];
        int c = s_cnt[src * a.El + l];
        if (c < 0 || off < 0 || off + c > a.maxr) {   // corrupt counts: skip, report
          atomicExch(status, (int)kErrBounds);
          c = 0;
        }
        for (int r = 0; r < c && n < max_items; r += bn, ++n) {
          items[n * 3 + 0] = l;
          items[n * 3 + 1] = src * a.maxr + off + r;
          items[n * 3 + 2] = min(bn, c - r);
        }
      }
    if (n >= max_items) atomicExch(status, (int)kErrBounds);
    s_n = n;
    int* nrows = reinterpret_cast<int*>(a.peer[a.rank] + kNRowsOff);
    for (int src = 0; src < a.world; ++src) {
      int tot = 0;
      for (int l = 0; l < a.El; ++l) tot += s_cnt[src * a.El + l];
      nrows[src] = (tot >= 0 && tot <= a.maxr) ? tot : 0;
    }
  }
  __syncthreads();
  for (int i = s_n + threadIdx.x; i < max_items; i += blockDim.x) {
    items[i * 3 + 0] = 0;
    items[i * 3 + 1] = 0;
    items[i * 3 + 2] = 0;
  }
}

// ---- 3b. SiLU(g) * u -> e4m3 rows, for the rows the work table covers only ---------------------
// gu bf16 [R, 2I]; one CTA (128 threads) per (item, row of the item)
__global__ void __launch_bounds__(128) silu_items_kernel(const __nv_bfloat16* __restrict__ gu,
                                                         int I, const int* __restrict__ items,
                                                         int bn, uint8_t* __restrict__ q,
                                                         float* __restrict__ scale) {
  __shared__ float red[4];
  pdl_wait();
  pdl_trigger();
  const int it = blockIdx.x / bn, j = blockIdx.x % bn;
  if (j >= items[it * 3 + 2]) return;
  const int row = items[it * 3 + 1] + j;
  const __nv_bfloat16* g = gu + (size_t)row * 2 * I;
  const __nv_bfloat16* u = g + I;
  float amax = 0.f;
  for (int i = threadIdx.x; i < I; i += blockDim.x) {
    const float gv = __bfloat162float(g[i]);
    const float v = bf16_round(gv / (1.f + __expf(-gv)) * __bfloat162float(u[i]));
    amax = fmaxf(amax, fabsf(v));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  const float sc = fmaxf(amax / 448.f, 1.f / (448.f * 512.f));
  const float inv = 1.f / sc;
  for (int i = threadIdx.x; i < I; i += blockDim.x) {
    const float gv = __bfloat162float(g[i]);
    const float v = bf16_round(gv / (1.f + __expf(-gv)) * __bfloat162float(u[i]));
    q[(size_t)row * I + i] = f32_to_e4m3(v * inv);
  }
  if (threadIdx.x == 0) scale[row] = sc;
}

// ---- 4. combine send ---------------------------------------------------------------------------
// y bf16 [world * maxr, H] (receive-row order); one warp per row
__global__ void __launch_bounds__(256) combine_send_kernel(const __grid_constant__ Args a,
                                                           const __nv_bfloat16* __restrict__ y,
                                                           int* __restrict__ status) {
  __shared__ int last;
  pdl_wait();
  pdl_trigger();
  const uint32_t e = seq_of(a);
  const uint8_t* me = a.peer[a.rank];
  const int* nrows = reinterpret_cast<const int*>(me + kNRowsOff);
  const int* meta = reinterpret_cast<const int*>(me + a.m_off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int R = a.world * a.maxr;
  for (int r = blockIdx.x * nw + warp; r < R; r += gridDim.x * nw) {
    const int src = r / a.maxr, slot = r % a.maxr;
    if (slot >= nrows[src]) continue;
    const int m = meta[r];
    if (m < 0 || m >= a.maxt * a.K) {
      if (lane == 0) atomicExch(status, (int)kErrBounds);
      continue;
    }
    const uint4* from = reinterpret_cast<const uint4*>(y + (size_t)r * a.H);
    uint4* to = reinterpret_cast<uint4*>(a.peer[src] + a.c_off + (int64_t)m * a.H * 2);
    for (int c = lane; c < a.H / 8; c += 32) to[c] = from[c];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* arrive = reinterpret_cast<uint32_t*>(a.peer[a.rank] + kArriveCombOff);
    last = atomicAdd(arrive, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence_system();
  if (threadIdx.x < a.world)
    st_release_sys(reinterpret_cast<uint32_t*>(a.peer[threadIdx.x] + kCombDoneOff) + a.rank, e);
  if (threadIdx.x == 0) *reinterpret_cast<uint32_t*>(a.peer[a.rank] + kArriveCombOff) = 0;
}

// ---- 5. combine reduce -------------------------------------------------------------------------
// out[t] = sum_k w[t, k] * comb[t * K + k]; grid over (token, 8-column chunks)
__global__ void __launch_bounds__(256) combine_reduce_kernel(const __grid_constant__ Args a,
                                                             const float* __restrict__ w, int T,
                                                             __nv_bfloat16* __restrict__ out,
                                                             int* __restrict__ status) {
  __shared__ int last;
  pdl_wait();
  pdl_trigger();
  const uint32_t e = seq_of(a);
  uint8_t* me = a.peer[a.rank];
  if (threadIdx.x < a.world)
    wait_flag_geq(reinterpret_cast<const uint32_t*>(me + kCombDoneOff) + threadIdx.x, e, status,
                  kErrPeerTimeout);
  __syncthreads();
  const __nv_bfloat16* comb = reinterpret_cast<const __nv_bfloat16*>(me + a.c_off);
  const int chunks = a.H / 8;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < T * chunks;
       i += gridDim.x * blockDim.x) {
    const int t = i / chunks, c = i % chunks;
    float acc[8] = {};
    for (int k = 0; k < a.K; ++k) {
      const float wk = w[t * a.K + k];
      const uint4 v =
          *reinterpret_cast<const uint4*>(comb + ((size_t)(t * a.K + k)) * a.H + c * 8);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        acc[2 * j] += wk * f.x;
        acc[2 * j + 1] += wk * f.y;
      }
    }
    uint4 o;
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) oh[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
    *reinterpret_cast<uint4*>(out + (size_t)t * a.H + c * 8) = o;
  }
  // the last CTA closes the call: the next call's flags carry the next sequence number
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* arrive = reinterpret_cast<uint32_t*>(me + kArriveRedOff);
    last = atomicAdd(arrive, 1u) == gridDim.x - 1;
    if (last) {
      *arrive = 0;
      *reinterpret_cast<volatile uint32_t*>(me + kEpochOff) = e;
    }
  }
}

}  // namespace ep

// ---- host ----------------------------------------------------------------------------------------
static ep::Args make_args(const std::vector<int64_t>& peers, int64_t rank, int64_t maxr,
                          int64_t H, int64_t K, int64_t El, int64_t maxt) {
  const int world = (int)peers.size();
  TORCH_CHECK(world >= 1 && world <= ep::kMaxWorld, "ep: world 1..8");
  TORCH_CHECK(H % 16 == 0 && El * world <= ep::kMaxExperts && K >= 1 && maxr >= 1 && maxt >= 1,
              "ep: H % 16, experts <= 256");
  ep::Args a = {};
  for (int i = 0; i < world; ++i) a.peer[i] = reinterpret_cast<uint8_t*>(peers[i]);
  a.world = world;
  a.rank = (int)rank;
  a.maxr = (int)maxr;
  a.maxt = (int)maxt;
  a.H = (int)H;
  a.K = (int)K;
  a.El = (int)El;
  const int64_t R = world * maxr;
  a.q_off = ep::kDataOff;
  a.s_off = a.q_off + ((R * H + 255) / 256) * 256;
  a.m_off = a.s_off + ((R * 4 + 255) / 256) * 256;
  a.c_off = a.m_off + ((R * 4 + 255) / 256) * 256;
  return a;
}

int64_t ep_buffer_bytes(int64_t world, int64_t maxr, int64_t H, int64_t K, int64_t maxt) {
  std::vector<int64_t> fake(world, 0);
  ep::Args a = make_args(fake, 0, maxr, H, K, 1, maxt);
  return a.c_off + maxt * K * H * 2;
}

// offsets of the receive rows / scales / meta and the combine buffer
std::vector<int64_t> ep_offsets(int64_t world, int64_t maxr, int64_t H, int64_t K, int64_t maxt) {
  std::vector<int64_t> fake(world, 0);
  ep::Args a = make_args(fake, 0, maxr, H, K, 1, maxt);
  return {a.q_off, a.s_off, a.m_off, a.c_off};
}

void ep_dispatch(std::vector<int64_t> peers, int64_t rank, int64_t maxr, int64_t El,
                 int64_t maxt, torch::Tensor q, torch::Tensor s, torch::Tensor ids,
                 torch::Tensor status) {
  const int T = q.size(0), H = q.size(1), K = ids.size(1);
  TORCH_CHECK(T >= 0 && T <= maxt && ids.size(0) == T && ids.scalar_type() == at::kInt &&
                  ids.is_contiguous(), "ep_dispatch: ids int32 [T <= maxt, K]");
  TORCH_CHECK(q.element_size() == 1 && q.stride(1) == 1 && q.stride(0) % 16 == 0 &&
                  (reinterpret_cast<uintptr_t>(q.data_ptr()) % 16) == 0 &&
                  s.scalar_type() == at::kFloat && s.numel() >= T, "ep_dispatch: q / s");
  TORCH_CHECK((int64_t)T * K <= maxr, "ep_dispatch: rows exceed a source segment");
  ep::Args a = make_args(peers, rank, maxr, H, K, El, maxt);
  const at::cuda::CUDAGuard guard(q.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int P = T * K, E = (int)El * a.world;
  const size_t smem = (size_t)(2 * P + 2 * E) * sizeof(int);
  TORCH_CHECK(smem <= 200 * 1024, "ep_dispatch: too many pairs");
  auto kern = ep::dispatch_kernel;
  C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)std::max<size_t>(smem, 48 * 1024)));
  const int ctas = std::max(1, std::min(32, (P + 15) / 16));
  C10_CUDA_CHECK(launch_pdl(kern, dim3(ctas), dim3(512), smem, stream, a,
                            (const uint8_t*)q.data_ptr(), (int)q.stride(0),
                            s.data_ptr<float>(), ids.data_ptr<int>(), T, status.data_ptr<int>()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ep_items(std::vector<int64_t> peers, int64_t rank, int64_t maxr, int64_t H, int64_t K,
              int64_t El, int64_t maxt, int64_t bn, torch::Tensor items, torch::Tensor status) {
  ep::Args a = make_args(peers, rank, maxr, H, K, El, maxt);
  TORCH_CHECK(items.scalar_type() == at::kInt && items.dim() == 2 && items.size(1) == 3 &&
                  items.is_contiguous(), "ep_items: items int32 [n, 3]");
  const at::cuda::CUDAGuard guard(items.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  C10_CUDA_CHECK(launch_pdl(ep::items_kernel, dim3(1), dim3(256), 0, stream, a, (int)bn,
                            items.data_ptr<int>(), (int)items.size(0), status.data_ptr<int>()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ep_silu_items(torch::Tensor gu, torch::Tensor items, int64_t bn, torch::Tensor q,
                   torch::Tensor scale) {
  const int I = gu.size(1) / 2;
  TORCH_CHECK(gu.scalar_type() == at::kBFloat16 && gu.is_contiguous() && q.is_contiguous() &&
                  q.element_size() == 1 && q.size(1) == I && q.size(0) == gu.size(0) &&
                  scale.scalar_type() == at::kFloat && scale.numel() >= gu.size(0),
              "ep_silu_items: shapes");
  const at::cuda::CUDAGuard guard(gu.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  C10_CUDA_CHECK(launch_pdl(ep::silu_items_kernel, dim3(items.size(0) * bn), dim3(128), 0,
                            stream, (const __nv_bfloat16*)gu.data_ptr(), I, items.data_ptr<int>(),
                            (int)bn, (uint8_t*)q.data_ptr(), scale.data_ptr<float>()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ep_combine(std::vector<int64_t> peers, int64_t rank, int64_t maxr, int64_t El,
                int64_t maxt, torch::Tensor y, torch::Tensor w, torch::Tensor out,
                torch::Tensor status) {
  const int H = y.size(1), T = w.size(0), K = w.size(1);
  ep::Args a = make_args(peers, rank, maxr, H, K, El, maxt);
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && y.is_contiguous() &&
                  y.size(0) == (int64_t)a.world * maxr, "ep_combine: y [world * maxr, H]");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous() && T <= maxt &&
                  out.scalar_type() == at::kBFloat16 && out.is_contiguous() &&
                  out.size(0) == T && out.size(1) == H, "ep_combine: w / out");
  const at::cuda::CUDAGuard guard(y.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  C10_CUDA_CHECK(launch_pdl(ep::combine_send_kernel, dim3(32), dim3(256), 0, stream, a,
                            (const __nv_bfloat16*)y.data_ptr(), status.data_ptr<int>()));
  const int blocks = std::max(1, std::min(64, (T * H / 8 + 255) / 256));
  C10_CUDA_CHECK(launch_pdl(ep::combine_reduce_kernel, dim3(blocks), dim3(256), 0, stream, a,
                            w.data_ptr<float>(), T, (__nv_bfloat16*)out.data_ptr(),
                            status.data_ptr<int>()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace rad
