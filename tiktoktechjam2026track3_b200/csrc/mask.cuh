// The harness's valid-token mask turned into what the kernels take, in one launch.
//
// generate_random_case (transformer_benchmark/cases.py:87-97) produces prefix masks: row b is true
// at positions < length_b. The attention kernels take the lengths (kv_len, keys >= kv_len[b] are
// padding: models.py:63-66) and the GEMM epilogues / final LayerNorm take the mask bytes as a row
// mask (padded rows zeroed: models.py:78-79, 736-737, 917-918). One block per sequence counts the
// row's true entries, checks that the row is a prefix of that length, writes the length, the
// row's verdict (1 = not a prefix) and, when asked, a copy of the row's bytes — the work of seven
// small tensor operations and two copies on the host path of every forward pass with a new mask.
#pragma once
#include "b2_common.cuh"

namespace b2 {

constexpr int kMaskThreads = 256;

__global__ void __launch_bounds__(kMaskThreads)
    mask_lengths_kernel(const uint8_t* __restrict__ mask, int64_t seq_len, int32_t* __restrict__ kv_len,
                        uint8_t* __restrict__ row_copy, uint8_t* __restrict__ not_prefix) {
  // No early launch of the dependent kernel: the attention kernels read kv_len in their prologue,
  // before their own wait for this grid, so the next launch starts only once this one has ended.
  pdl_wait_previous_grid();
  __shared__ int warp_sums[kMaskThreads / 32];
  __shared__ int warp_bad[kMaskThreads / 32];
  const int64_t b = blockIdx.x;
  const uint8_t* row = mask + b * seq_len;
  int count = 0;
  for (int64_t s = threadIdx.x; s < seq_len; s += kMaskThreads) count += row[s] != 0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) count += __shfl_xor_sync(0xffffffffu, count, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) warp_sums[warp] = count;
  __syncthreads();
  int len = 0;
#pragma unroll
  for (int w = 0; w < kMaskThreads / 32; ++w) len += warp_sums[w];
  // Prefix check: entry s must be true exactly when s < len.
  int bad = 0;
  for (int64_t s = threadIdx.x; s < seq_len; s += kMaskThreads) {
    const uint8_t v = row[s];
    bad |= (v != 0) != (s < len);
    if (row_copy != nullptr) row_copy[b * seq_len + s] = v != 0 ? 1 : 0;
  }
  bad = __any_sync(0xffffffffu, bad) ? 1 : 0;
  if (lane == 0) warp_bad[warp] = bad;
  __syncthreads();
  if (threadIdx.x == 0) {
    int any = 0;
#pragma unroll
    for (int w = 0; w < kMaskThreads / 32; ++w) any |= warp_bad[w];
    kv_len[b] = len;
    not_prefix[b] = static_cast<uint8_t>(any);
  }
}

cudaError_t launch_mask_lengths(const uint8_t* mask, int64_t batch, int64_t seq_len, int32_t* kv_len,
                                uint8_t* row_copy, uint8_t* not_prefix, cudaStream_t stream) {
  return launch_pdl(mask_lengths_kernel, dim3(static_cast<unsigned>(batch)), dim3(kMaskThreads), 0, stream, mask,
                    seq_len, kv_len, row_copy, not_prefix);
}

}  // namespace b2
