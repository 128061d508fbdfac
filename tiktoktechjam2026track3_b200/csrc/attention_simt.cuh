// Attention forward on CUDA cores for the head dims the tensor-core kernel does not tile
// (8, 16, 32, 256: the reference's official case matrix, transformer_benchmark/cases.py:42-57,
// uses 8, 32 and 256 at D = 32..1024 and S = 32..1024). Same contract as the tensor-core path
// (BaselineSelfAttention.forward, models.py:55-75; masks as in attention.cuh): fp32 scores,
// online softmax in fp32, context written as bf16 into the token-major [B*S, H*hd] rows.
//
// Block = 128 threads over (b, h, a run of queries); TPQ = max(1, hd / 32) consecutive threads
// share a query, each holding hd / TPQ (<= 32) of its dims of q and of the output in registers
// (4-dim groups interleaved over the TPQ threads, so their shared-memory reads of a key row are
// consecutive 16-byte pieces, free of bank conflicts), so a score is a TPQ-wide shuffle reduction
// of partial dot products. Keys and values stream through shared memory in chunks, converted to
// fp32 once when staged (16-byte loads; the whole block shares a chunk), so the inner loop is
// 16-byte broadcast loads and FMAs only — converting bf16 at every use cost as many instructions
// as the FMAs. The running maximum is per query and, as in the tensor-core kernel, moves only
// when a score exceeds it by more than 2^8 (exp2 units), which keeps the rescale branch rare.
#pragma once
#include "b2_common.cuh"

namespace b2 {

template <int HD>
struct AttnSimtCfg {
  static constexpr int kThreads = 128;
  static constexpr int kTPQ = HD <= 32 ? 1 : HD / 32;  // threads per query
  static constexpr int kDPT = HD / kTPQ;               // dims per thread
  static constexpr int kQPB = kThreads / kTPQ;         // queries per block
  static constexpr int kChunk = HD >= 256 ? 32 : 64;   // keys per shared-memory chunk
  static constexpr int kSmemBytes = 2 * kChunk * HD * 4;  // fp32 K and V
  static_assert(HD % 8 == 0 && kDPT <= 32 && kDPT % 4 == 0 && (kTPQ & (kTPQ - 1)) == 0, "head_dim");
};

template <int HD>
__global__ void __launch_bounds__(128) attention_simt_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t ld_qkv,
                                                             AttnParams p) {
  using Cfg = AttnSimtCfg<HD>;
  extern __shared__ __align__(16) uint8_t simt_smem[];
  float* sk = reinterpret_cast<float*>(simt_smem);
  float* sv = sk + Cfg::kChunk * HD;
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
  // Float4 group i of this thread holds dims 4 (i TPQ + sub) .. +3.
  auto dim_of = [&](int i) { return (i * Cfg::kTPQ + sub) * 4; };
  const int64_t row_base = static_cast<int64_t>(b) * p.S;
  const bool live = qi < q_end;
  const int limit = p.causal ? min(kv_len, qi + 1) : kv_len;
  // Keys the block needs: up to the last query's causal limit.
  const int q_last = min(q0 + Cfg::kQPB, q_end) - 1;
  const int block_keys = p.causal ? min(kv_len, q_last + 1) : kv_len;
  constexpr float kRescaleThreshold = 8.0f;  // exp2 units

  float q[Cfg::kDPT], o[Cfg::kDPT];
  if (live) {
    const __nv_bfloat16* qp = qkv + (row_base + qi) * ld_qkv + p.q_col + h * HD;
#pragma unroll
    for (int i = 0; i < Cfg::kDPT / 4; ++i) {
      const uint2 raw = *reinterpret_cast<const uint2*>(qp + dim_of(i));
      const __nv_bfloat162* hv = reinterpret_cast<const __nv_bfloat162*>(&raw);
      q[4 * i] = __low2float(hv[0]) * p.scale_log2;
      q[4 * i + 1] = __high2float(hv[0]) * p.scale_log2;
      q[4 * i + 2] = __low2float(hv[1]) * p.scale_log2;
      q[4 * i + 3] = __high2float(hv[1]) * p.scale_log2;
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
      const uint4 kraw = *reinterpret_cast<const uint4*>(base + p.k_col);
      const uint4 vraw = *reinterpret_cast<const uint4*>(base + p.v_col);
      const __nv_bfloat162* kh = reinterpret_cast<const __nv_bfloat162*>(&kraw);
      const __nv_bfloat162* vh = reinterpret_cast<const __nv_bfloat162*>(&vraw);
      float4* kd = reinterpret_cast<float4*>(sk + key * HD + col);
      float4* vd = reinterpret_cast<float4*>(sv + key * HD + col);
      kd[0] = make_float4(__low2float(kh[0]), __high2float(kh[0]), __low2float(kh[1]), __high2float(kh[1]));
      kd[1] = make_float4(__low2float(kh[2]), __high2float(kh[2]), __low2float(kh[3]), __high2float(kh[3]));
      vd[0] = make_float4(__low2float(vh[0]), __high2float(vh[0]), __low2float(vh[1]), __high2float(vh[1]));
      vd[1] = make_float4(__low2float(vh[2]), __high2float(vh[2]), __low2float(vh[3]), __high2float(vh[3]));
    }
    __syncthreads();
    // Two keys per step: their dot products and V rows are independent, so one key's shared-memory
    // loads overlap the other's FMAs (the single-key chain was bound by shared-memory latency).
    for (int kk = 0; kk < n; kk += 2) {
      const bool has_b = kk + 1 < n;  // uniform across the block
      const float* kra = sk + kk * HD;
      const float* krb = kra + HD;
      float sa0 = 0.f, sa1 = 0.f, sb0 = 0.f, sb1 = 0.f;
#pragma unroll
      for (int i = 0; i < Cfg::kDPT / 4; ++i) {
        const float4 ka = *reinterpret_cast<const float4*>(kra + dim_of(i));
        sa0 = fmaf(q[4 * i], ka.x, sa0);
        sa1 = fmaf(q[4 * i + 1], ka.y, sa1);
        sa0 = fmaf(q[4 * i + 2], ka.z, sa0);
        sa1 = fmaf(q[4 * i + 3], ka.w, sa1);
        if (has_b) {
          const float4 kb = *reinterpret_cast<const float4*>(krb + dim_of(i));
          sb0 = fmaf(q[4 * i], kb.x, sb0);
          sb1 = fmaf(q[4 * i + 1], kb.y, sb1);
          sb0 = fmaf(q[4 * i + 2], kb.z, sb0);
          sb1 = fmaf(q[4 * i + 3], kb.w, sb1);
        }
      }
      float sa = sa0 + sa1, sb = sb0 + sb1;
#pragma unroll
      for (int off = Cfg::kTPQ / 2; off > 0; off >>= 1) {
        sa += __shfl_xor_sync(0xffffffffu, sa, off);
        sb += __shfl_xor_sync(0xffffffffu, sb, off);
      }
      // Masked keys (uniform across a query's threads); the causal limit masks a suffix.
      const bool va = c0 + kk < limit;
      const bool vb = has_b && c0 + kk + 1 < limit;
      if (!va) continue;
      const float mx = vb ? fmaxf(sa, sb) : sa;
      if (mx > m + kRescaleThreshold) {
        const float alpha = fast_exp2(m - mx);  // 0 on the first key (m = -inf)
        m = mx;
        l *= alpha;
#pragma unroll
        for (int i = 0; i < Cfg::kDPT; ++i) o[i] *= alpha;
      }
      const float pa = fast_exp2(sa - m);
      const float pb = vb ? fast_exp2(sb - m) : 0.f;
      l += pa + pb;
      const float* vra = sv + kk * HD;
      const float* vrb = vra + HD;
#pragma unroll
      for (int i = 0; i < Cfg::kDPT / 4; ++i) {
        const float4 va4 = *reinterpret_cast<const float4*>(vra + dim_of(i));
        o[4 * i] = fmaf(pa, va4.x, o[4 * i]);
        o[4 * i + 1] = fmaf(pa, va4.y, o[4 * i + 1]);
        o[4 * i + 2] = fmaf(pa, va4.z, o[4 * i + 2]);
        o[4 * i + 3] = fmaf(pa, va4.w, o[4 * i + 3]);
        if (vb) {
          const float4 vb4 = *reinterpret_cast<const float4*>(vrb + dim_of(i));
          o[4 * i] = fmaf(pb, vb4.x, o[4 * i]);
          o[4 * i + 1] = fmaf(pb, vb4.y, o[4 * i + 1]);
          o[4 * i + 2] = fmaf(pb, vb4.z, o[4 * i + 2]);
          o[4 * i + 3] = fmaf(pb, vb4.w, o[4 * i + 3]);
        }
      }
    }
  }
  if (!live) return;
  const float inv = l > 0.f ? 1.0f / l : 0.f;
  __nv_bfloat16* dst = p.ctx + (row_base + qi) * p.ld_ctx + h * HD;
#pragma unroll
  for (int i = 0; i < Cfg::kDPT / 4; ++i)
    *reinterpret_cast<uint2*>(dst + dim_of(i)) =
        make_uint2(pack_bf16x2(o[4 * i] * inv, o[4 * i + 1] * inv), pack_bf16x2(o[4 * i + 2] * inv, o[4 * i + 3] * inv));
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
