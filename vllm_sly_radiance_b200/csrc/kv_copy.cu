// Segment gather / scatter between the paged caches and one contiguous staging buffer, the copy
// engine of the KV offload tier.
//
// Reference behaviour: the offloading connector's GPU <-> CPU block transfers (vLLM
// OffloadingConnector as configured by kv-cache/README.md:1-60, with the reference's fixes for
// hybrid groups and mamba strides).  A cached item is one KV block (its page in every attention
// layer's K and V cache) or one GDN state slot (its conv + SSM state in every GDN layer): tens of
// segments spread over as many tensors.  Copying them one by one costs a DMA set-up per segment;
// here one launch packs all segments of a batch of items into a contiguous device staging buffer
// (or unpacks it), and the host tier moves each item with a single large copy.
//
// table: int64 [T, 3] = (base address, item stride in bytes, segment bytes) per cache tensor;
// offs: int64 [T] = offset of tensor t's segment inside an item of the staging buffer;
// idx: int32 [n] = item indices (block ids or slot ids).  Every address, stride, size and offset
// is a multiple of 16 bytes (checked on the host), so the copy moves 16-byte vectors.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace rad {
namespace kvc {

// blockIdx.y = item * T + t; blockIdx.x strides over the segment's 16-byte vectors
template <bool GATHER>
__global__ void __launch_bounds__(256) seg_copy_kernel(const int64_t* __restrict__ table,
                                                       const int64_t* __restrict__ offs,
                                                       const int* __restrict__ idx, int T,
                                                       uint8_t* __restrict__ stage,
                                                       int64_t item_bytes) {
  pdl_wait();
  pdl_trigger();
  const int it = blockIdx.y / T, t = blockIdx.y % T;
  const int64_t base = table[3 * t], stride = table[3 * t + 1], bytes = table[3 * t + 2];
  uint4* cache = reinterpret_cast<uint4*>(base + (int64_t)idx[it] * stride);
  uint4* st = reinterpret_cast<uint4*>(stage + (int64_t)it * item_bytes + offs[t]);
  const int64_t nv = bytes / 16;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nv;
       v += (int64_t)gridDim.x * blockDim.x) {
    if (GATHER) st[v] = cache[v];
    else cache[v] = st[v];
  }
}

}  // namespace kvc

// gather = true: cache segments of items idx -> stage [n, item_bytes]; false: the reverse
void segment_copy(torch::Tensor table, torch::Tensor offs, torch::Tensor idx, torch::Tensor stage,
                  int64_t item_bytes, bool gather) {
  TORCH_CHECK(table.is_cuda() && table.scalar_type() == at::kLong && table.dim() == 2 &&
                  table.size(1) == 3, "segment_copy: table int64 [T, 3] on the device");
  TORCH_CHECK(offs.is_cuda() && offs.scalar_type() == at::kLong && offs.numel() == table.size(0),
              "segment_copy: offs");
  TORCH_CHECK(idx.is_cuda() && idx.scalar_type() == at::kInt, "segment_copy: idx int32");
  TORCH_CHECK(stage.is_cuda() && stage.is_contiguous() && item_bytes % 16 == 0 &&
                  (reinterpret_cast<uintptr_t>(stage.data_ptr()) % 16) == 0 &&
                  stage.numel() >= idx.numel() * item_bytes, "segment_copy: stage");
  const int T = table.size(0), n = idx.numel();
  if (n == 0 || T == 0) return;
  TORCH_CHECK((int64_t)n * T < 65536, "segment_copy: too many segments per launch");
  const at::cuda::CUDAGuard guard(stage.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const dim3 grid(16, n * T);
  if (gather)
    C10_CUDA_CHECK(launch_pdl(kvc::seg_copy_kernel<true>, grid, dim3(256), 0, stream,
                              (const int64_t*)table.data_ptr(), (const int64_t*)offs.data_ptr(),
                              (const int*)idx.data_ptr(), T, (uint8_t*)stage.data_ptr(),
                              item_bytes));
  else
    C10_CUDA_CHECK(launch_pdl(kvc::seg_copy_kernel<false>, grid, dim3(256), 0, stream,
                              (const int64_t*)table.data_ptr(), (const int64_t*)offs.data_ptr(),
                              (const int*)idx.data_ptr(), T, (uint8_t*)stage.data_ptr(),
                              item_bytes));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace rad
