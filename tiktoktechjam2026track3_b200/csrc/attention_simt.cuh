// Attention forward on CUDA cores for the head dims the tensor-core kernel does not tile
// (8, 16, 32, 256: the reference's official case matrix, transformer_benchmark/cases.py:42-57,
// uses 8, 32 and 256 at D = 32..1024 and S = 32..1024). Same contract as the tensor-core path
// (BaselineSelfAttention.forward, models.py:55-75; masks as in attention.cuh): fp32 scores,
// online softmax in fp32, context written as bf16 into the token-major [B*S, H*hd] rows.
//
// Block = 128 threads over (b, h, a run of queries); TPQ = max(1, hd / 32) consecutive threads
// share a query, each holding hd / TPQ (<= 32) of its dims of q and of the output in registers,
// so a score is a TPQ-wide shuffle reduction of partial dot products. Keys and values stream
// through shared memory in chunks of 64 keys (16-byte loads; the whole block shares a chunk).
// The running maximum is per query; the output is rescaled only when it moves.
#pragma once
#include "b2_common.cuh"

namespace b2 {

template <int HD>
struct AttnSimtCfg {
  static constexpr int kThreads = 128;
  static constexpr int kTPQ = HD <= 32 ? 1 : HD / 32;  // threads per query
  static constexpr int kDPT = HD / kTPQ;               // dims per thread
  static constexpr int kQPB = kThreads / kTPQ;         // queries per block
  static constexpr int kChunk = 64;                    // keys per shared-memory chunk
  static constexpr int kSmemBytes = 2 * kChunk * HD * 2;
  static_assert(HD % 8 == 0 && kDPT <= 32 && (kTPQ & (kTPQ - 1)) == 0, "head_dim");
};

template <int HD>
__global__ void __launch_bounds__(128) attention_simt_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t ld_qkv,
                                                             AttnParams p) {
  using Cfg = AttnSimtCfg<HD>;
  extern __shared__ __align__(16) uint8_t simt_smem[];
  __nv_bfloat16* sk = reinterpret_cast<__nv_bfloat16*>(simt_smem);
  __nv_bfloat16* sv = sk + Cfg::kChunk * HD;
  pdl_wait_previous_grid();
  pdl_allow_next_grid();

  const int b = blockIdx.x / p.H;
  const int h = blockIdx.x % p.H;
  const int range_blocks[2] = {(p.q_end[0] - p.q_tile0[0] * 128 + Cfg::kQPB - 1) / Cfg::kQPB,
                               (p.q_end[1] - p.q_tile0[1] * 128 + Cfg::kQPB - 1) / Cfg::kQPB};
  int y_local;
  const int rg = attn_range_of(p, static_cast<int>(blockIdx.y), range_blocks, y_local);
  const int q_end = p.q_end[rg];
  const int q0 = p.q_tile0[rg] * 128 + y_local * Cfg::kQPB;
  const int kv_len = p.kv_len != nullptr ? p.kv_len[b] : p.S;
  const int qi = q0 + static_cast<int>(threadIdx.x) / Cfg::kTPQ;
  const int sub = static_cast<int>(threadIdx.x) % Cfg::kTPQ;
  const int d0 = sub * Cfg::kDPT;
  const int64_t row_base = static_cast<int64_t>(b) * p.S;
  const bool live = qi < q_end;
  const int limit = p.causal ? min(kv_len, qi + 1) : kv_len;
  // Keys the block needs: up to the last query's causal limit.
  const int q_last = min(q0 + Cfg::kQPB, q_end) - 1;
  const int block_keys = p.causal ? min(kv_len, q_last + 1) : kv_len;

  float q[Cfg::kDPT], o[Cfg::kDPT];
  if (live) {
    const __nv_bfloat16* qp = qkv + (row_base + qi) * ld_qkv + p.q_col + h * HD + d0;
#pragma unroll
    for (int i = 0; i < Cfg::kDPT; i += 8) {
      const uint4 raw = *reinterpret_cast<const uint4*>(qp + i);
      const __nv_bfloat162* hv = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        q[i + 2 * k] = __low2float(hv[k]) * p.scale_log2;
        q[i + 2 * k + 1] = __high2float(hv[k]) * p.scale_log2;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < Cfg::kDPT; ++i) q[i] = 0.f;
  }
#pragma unroll
  for (int i = 0; i < Cfg::kDPT; ++i) o[i] = 0.f;
  float m = -INFINITY, l = 0.f;

  for (int c0 = 0; c0 < block_keys; c0 += Cfg::kChunk) {
    const int n = min(Cfg::kChunk, block_keys - c0);
    __syncthreads();  // the previous chunk is no longer read
    constexpr int kVecPerRow = HD / 8;
    for (int idx = threadIdx.x; idx < n * kVecPerRow; idx += Cfg::kThreads) {
      const int key = idx / kVecPerRow;
      const int col = (idx % kVecPerRow) * 8;
      const __nv_bfloat16* base = qkv + (row_base + c0 + key) * ld_qkv + h * HD + col;
      *reinterpret_cast<uint4*>(sk + key * HD + col) = *reinterpret_cast<const uint4*>(base + p.k_col);
      *reinterpret_cast<uint4*>(sv + key * HD + col) = *reinterpret_cast<const uint4*>(base + p.v_col);
    }
    __syncthreads();
    for (int kk = 0; kk < n; ++kk) {
      const __nv_bfloat16* kr = sk + kk * HD + d0;
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < Cfg::kDPT; i += 2) {
        const float2 kf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(kr + i));
        s = fmaf(q[i], kf.x, s);
        s = fmaf(q[i + 1], kf.y, s);
      }
#pragma unroll
      for (int off = Cfg::kTPQ / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      if (c0 + kk >= limit) continue;  // masked key (uniform across the query's threads)
      if (s > m) {
        const float alpha = fast_exp2(m - s);  // 0 on the first key (m = -inf)
        m = s;
        l *= alpha;
#pragma unroll
        for (int i = 0; i < Cfg::kDPT; ++i) o[i] *= alpha;
      }
      const float pr = fast_exp2(s - m);
      l += pr;
      const __nv_bfloat16* vr = sv + kk * HD + d0;
#pragma unroll
      for (int i = 0; i < Cfg::kDPT; i += 2) {
        const float2 vf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(vr + i));
        o[i] = fmaf(pr, vf.x, o[i]);
        o[i + 1] = fmaf(pr, vf.y, o[i + 1]);
      }
    }
  }
  if (!live) return;
  const float inv = l > 0.f ? 1.0f / l : 0.f;
  __nv_bfloat16* dst = p.ctx + (row_base + qi) * p.ld_ctx + h * HD + d0;
#pragma unroll
  for (int i = 0; i < Cfg::kDPT; i += 8)
    *reinterpret_cast<uint4*>(dst + i) = make_uint4(pack_bf16x2(o[i] * inv, o[i + 1] * inv),
                                                    pack_bf16x2(o[i + 2] * inv, o[i + 3] * inv),
                                                    pack_bf16x2(o[i + 4] * inv, o[i + 5] * inv),
                                                    pack_bf16x2(o[i + 6] * inv, o[i + 7] * inv));
}

template <int HD>
static cudaError_t launch_attention_simt(const __nv_bfloat16* qkv, int64_t ld_qkv, const AttnParams& p,
                                         cudaStream_t stream) {
  using Cfg = AttnSimtCfg<HD>;
  if (Cfg::kSmemBytes > 48 * 1024) {
    static std::once_flag once[64];
    int dev = 0;
    cudaGetDevice(&dev);
    cudaError_t attr_err = cudaSuccess;
    std::call_once(once[dev & 63], [&] {
      attr_err = cudaFuncSetAttribute(attention_simt_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      Cfg::kSmemBytes);
    });
    if (attr_err != cudaSuccess) return attr_err;
  }
  unsigned rows = 0;
  for (int r = 0; r < p.n_ranges; ++r) rows += (p.q_end[r] - p.q_tile0[r] * 128 + Cfg::kQPB - 1) / Cfg::kQPB;
  dim3 grid(p.B * p.H, rows);
  return launch_pdl(attention_simt_kernel<HD>, grid, dim3(Cfg::kThreads), Cfg::kSmemBytes, stream, qkv, ld_qkv, p);
}

}  // namespace b2
