// LayerNorm over the last dimension, fp32 statistics, bf16 output.
//
// Semantics follow nn.LayerNorm(D, eps) as BaselineTransformerBlock applies it
// (transformer_benchmark/models.py:721,723 for norm1/norm2 and :907 for final_norm):
//   y = (x - mean) / sqrt(var + eps) * gamma + beta,  var biased (divide by D).
// The padded-row zeroing that BaselineTransformer.forward applies after the final norm
// (models.py:917-918) is fused here: rows whose row_mask byte is 0 are written as zeros.
//
// Input is the fp32 residual stream, or the bf16 model input (first norm of the first block); in
// the bf16 case the kernel also writes the fp32 copy that seeds the residual stream.
//
// One warp per row, values held in registers, 16-byte loads / 8-byte stores, so each element
// is read once and written once: the kernel is HBM-bound at 6 (fp32 in) or 8 (bf16 in + fp32
// copy + bf16 out) bytes per element.
#pragma once
#include "b2_common.cuh"

namespace b2 {

constexpr int kLnWarpsPerBlock = 8;

template <int NV, bool kInBf16>
__global__ void __launch_bounds__(kLnWarpsPerBlock * 32)
    layernorm_vec_kernel(const void* __restrict__ x_, const __nv_bfloat16* __restrict__ gamma,
                         const __nv_bfloat16* __restrict__ beta, float eps, __nv_bfloat16* __restrict__ y,
                         float* __restrict__ resid_out, const uint8_t* __restrict__ row_mask, int64_t rows) {
  constexpr int D = NV * 128;
  const int lane = threadIdx.x & 31;
  // gamma and beta are parameters, never written by the kernel this launch waits for: up to
  // D = 2048 they are loaded before the programmatic-dependent-launch wait, so their latency
  // overlaps the previous kernel's tail instead of following the row reductions (wider rows load
  // them after the reductions, keeping the registers for the row).
  constexpr bool kEarly = NV <= 16;
  const uint2* gr = reinterpret_cast<const uint2*>(gamma);
  const uint2* br = reinterpret_cast<const uint2*>(beta);
  uint2 graw[NV], braw[NV];
  if constexpr (kEarly) {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      graw[i] = __ldg(gr + i * 32 + lane);
      braw[i] = __ldg(br + i * 32 + lane);
    }
  }
  pdl_wait_previous_grid();
  pdl_allow_next_grid();
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kLnWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;

  float v[NV][4];
  if constexpr (kInBf16) {
    const uint2* xr = reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(x_) + row * D);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      uint2 raw = __ldg(xr + i * 32 + lane);
      __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&raw.x);
      __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&raw.y);
      v[i][0] = __low2float(a);
      v[i][1] = __high2float(a);
      v[i][2] = __low2float(b);
      v[i][3] = __high2float(b);
    }
    if (resid_out != nullptr) {
      float4* rr = reinterpret_cast<float4*>(resid_out + row * D);
#pragma unroll
      for (int i = 0; i < NV; ++i) rr[i * 32 + lane] = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
    }
  } else {
    const float4* xr = reinterpret_cast<const float4*>(static_cast<const float*>(x_) + row * D);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float4 t = __ldg(xr + i * 32 + lane);
      v[i][0] = t.x;
      v[i][1] = t.y;
      v[i][2] = t.z;
      v[i][3] = t.w;
    }
  }

  uint2* yr = reinterpret_cast<uint2*>(y + row * D);
  if (row_mask != nullptr && row_mask[row] == 0) {
#pragma unroll
    for (int i = 0; i < NV; ++i) yr[i * 32 + lane] = make_uint2(0u, 0u);
    return;
  }

  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) s += (v[i][0] + v[i][1]) + (v[i][2] + v[i][3]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s * (1.0f / D);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float d = v[i][j] - mean;
      q = fmaf(d, d, q);
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float rstd = rsqrtf(q * (1.0f / D) + eps);

#pragma unroll
  for (int i = 0; i < NV; ++i) {
    if constexpr (!kEarly) {
      graw[i] = __ldg(gr + i * 32 + lane);
      braw[i] = __ldg(br + i * 32 + lane);
    }
    __nv_bfloat162 g0 = *reinterpret_cast<__nv_bfloat162*>(&graw[i].x);
    __nv_bfloat162 g1 = *reinterpret_cast<__nv_bfloat162*>(&graw[i].y);
    __nv_bfloat162 b0 = *reinterpret_cast<__nv_bfloat162*>(&braw[i].x);
    __nv_bfloat162 b1 = *reinterpret_cast<__nv_bfloat162*>(&braw[i].y);
    const float o0 = fmaf((v[i][0] - mean) * rstd, __low2float(g0), __low2float(b0));
    const float o1 = fmaf((v[i][1] - mean) * rstd, __high2float(g0), __high2float(b0));
    const float o2 = fmaf((v[i][2] - mean) * rstd, __low2float(g1), __low2float(b1));
    const float o3 = fmaf((v[i][3] - mean) * rstd, __high2float(g1), __high2float(b1));
    yr[i * 32 + lane] = make_uint2(pack_bf16x2(o0, o1), pack_bf16x2(o2, o3));
  }
}

// Any D: one warp per row, three strided passes over the row (sum, squared deviations,
// normalise). Used only for widths that are not a multiple of 128.
template <bool kInBf16>
__global__ void __launch_bounds__(kLnWarpsPerBlock * 32)
    layernorm_any_kernel(const void* __restrict__ x_, const __nv_bfloat16* __restrict__ gamma,
                         const __nv_bfloat16* __restrict__ beta, float eps, __nv_bfloat16* __restrict__ y,
                         float* __restrict__ resid_out, const uint8_t* __restrict__ row_mask, int64_t rows,
                         int64_t D) {
  pdl_wait_previous_grid();
  pdl_allow_next_grid();
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kLnWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;
  auto load = [&](int64_t c) -> float {
    if constexpr (kInBf16)
      return __bfloat162float(static_cast<const __nv_bfloat16*>(x_)[row * D + c]);
    else
      return static_cast<const float*>(x_)[row * D + c];
  };
  if (kInBf16 && resid_out != nullptr)
    for (int64_t c = lane; c < D; c += 32) resid_out[row * D + c] = load(c);
  if (row_mask != nullptr && row_mask[row] == 0) {
    for (int64_t c = lane; c < D; c += 32) y[row * D + c] = __float2bfloat16_rn(0.f);
    return;
  }
  float s = 0.f;
  for (int64_t c = lane; c < D; c += 32) s += load(c);
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / static_cast<float>(D);
  float q = 0.f;
  for (int64_t c = lane; c < D; c += 32) {
    const float d = load(c) - mean;
    q = fmaf(d, d, q);
  }
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float rstd = rsqrtf(q / static_cast<float>(D) + eps);
  for (int64_t c = lane; c < D; c += 32) {
    const float o = fmaf((load(c) - mean) * rstd, __bfloat162float(gamma[c]), __bfloat162float(beta[c]));
    y[row * D + c] = __float2bfloat16_rn(o);
  }
}

// Residual update fused with the LayerNorm that follows it (tensor-parallel blocks, where the
// GEMM epilogue cannot add the residual because the projection output is a per-rank partial sum
// that is all-reduced first):
//   r      = row kept ? r + delta + bias : (kZeroRows ? 0 : r)      (written back, fp32)
//   y      = LayerNorm(r) in bf16, or 0 for masked rows when kZeroY
// kZeroRows reproduces the block's final masked_fill (models.py:736-737); kZeroY the one after
// final_norm (models.py:917-918). Masked rows keep x + 0 after attention (models.py:78-79, :733).
template <int NV, bool kZeroRows, bool kZeroY>
__global__ void __launch_bounds__(kLnWarpsPerBlock * 32)
    add_layernorm_vec_kernel(float* __restrict__ resid, const float* __restrict__ delta,
                             const __nv_bfloat16* __restrict__ bias, const uint8_t* __restrict__ row_mask,
                             const __nv_bfloat16* __restrict__ gamma, const __nv_bfloat16* __restrict__ beta,
                             float eps, __nv_bfloat16* __restrict__ y, int64_t rows) {
  pdl_wait_previous_grid();
  pdl_allow_next_grid();
  constexpr int D = NV * 128;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kLnWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;
  const bool keep = row_mask == nullptr || row_mask[row] != 0;
  float4* rr = reinterpret_cast<float4*>(resid + row * D);
  const float4* dr = reinterpret_cast<const float4*>(delta + row * D);
  float v[NV][4];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    float4 r = rr[i * 32 + lane];
    if (keep) {
      const float4 dd = __ldg(dr + i * 32 + lane);
      float b[4] = {0.f, 0.f, 0.f, 0.f};
      if (bias != nullptr) {
        uint2 braw = __ldg(reinterpret_cast<const uint2*>(bias) + i * 32 + lane);
        __nv_bfloat162 b0 = *reinterpret_cast<__nv_bfloat162*>(&braw.x);
        __nv_bfloat162 b1 = *reinterpret_cast<__nv_bfloat162*>(&braw.y);
        b[0] = __low2float(b0);
        b[1] = __high2float(b0);
        b[2] = __low2float(b1);
        b[3] = __high2float(b1);
      }
      r.x += dd.x + b[0];
      r.y += dd.y + b[1];
      r.z += dd.z + b[2];
      r.w += dd.w + b[3];
      rr[i * 32 + lane] = r;
    } else if (kZeroRows) {
      r = make_float4(0.f, 0.f, 0.f, 0.f);
      rr[i * 32 + lane] = r;
    }
    v[i][0] = r.x;
    v[i][1] = r.y;
    v[i][2] = r.z;
    v[i][3] = r.w;
  }
  uint2* yr = reinterpret_cast<uint2*>(y + row * D);
  if (kZeroY && !keep) {
#pragma unroll
    for (int i = 0; i < NV; ++i) yr[i * 32 + lane] = make_uint2(0u, 0u);
    return;
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) s += (v[i][0] + v[i][1]) + (v[i][2] + v[i][3]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s * (1.0f / D);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float d = v[i][j] - mean;
      q = fmaf(d, d, q);
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float rstd = rsqrtf(q * (1.0f / D) + eps);
  const uint2* gr = reinterpret_cast<const uint2*>(gamma);
  const uint2* br = reinterpret_cast<const uint2*>(beta);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    uint2 graw = __ldg(gr + i * 32 + lane);
    uint2 braw = __ldg(br + i * 32 + lane);
    __nv_bfloat162 g0 = *reinterpret_cast<__nv_bfloat162*>(&graw.x);
    __nv_bfloat162 g1 = *reinterpret_cast<__nv_bfloat162*>(&graw.y);
    __nv_bfloat162 b0 = *reinterpret_cast<__nv_bfloat162*>(&braw.x);
    __nv_bfloat162 b1 = *reinterpret_cast<__nv_bfloat162*>(&braw.y);
    const float o0 = fmaf((v[i][0] - mean) * rstd, __low2float(g0), __low2float(b0));
    const float o1 = fmaf((v[i][1] - mean) * rstd, __high2float(g0), __high2float(b0));
    const float o2 = fmaf((v[i][2] - mean) * rstd, __low2float(g1), __low2float(b1));
    const float o3 = fmaf((v[i][3] - mean) * rstd, __high2float(g1), __high2float(b1));
    yr[i * 32 + lane] = make_uint2(pack_bf16x2(o0, o1), pack_bf16x2(o2, o3));
  }
}

template <bool kZeroRows, bool kZeroY>
static cudaError_t launch_add_layernorm_t(float* resid, const float* delta, const __nv_bfloat16* bias,
                                          const uint8_t* row_mask, const __nv_bfloat16* gamma,
                                          const __nv_bfloat16* beta, float eps, __nv_bfloat16* y, int64_t rows,
                                          int64_t D, cudaStream_t stream) {
  const dim3 block(kLnWarpsPerBlock * 32);
  const dim3 grid(static_cast<unsigned>((rows + kLnWarpsPerBlock - 1) / kLnWarpsPerBlock));
#define B2_ALN_CASE(NV)                                                                                          \
  case NV:                                                                                                       \
    return launch_pdl(add_layernorm_vec_kernel<NV, kZeroRows, kZeroY>, grid, block, 0, stream, resid, delta, bias, \
                      row_mask, gamma, beta, eps, y, rows);
  switch (D / 128) {
    B2_ALN_CASE(1)
    B2_ALN_CASE(2)
    B2_ALN_CASE(4)
    B2_ALN_CASE(6)
    B2_ALN_CASE(8)
    B2_ALN_CASE(16)
    B2_ALN_CASE(32)
    default:
      return cudaErrorInvalidValue;
  }
#undef B2_ALN_CASE
}

// Widths the fused residual + LayerNorm kernel is instantiated for (D = 128 * NV).
inline bool add_layernorm_supported(int64_t D) {
  if (D % 128 != 0) return false;
  switch (D / 128) {
    case 1: case 2: case 4: case 6: case 8: case 16: case 32:
      return true;
    default:
      return false;
  }
}

cudaError_t launch_add_layernorm(float* resid, const float* delta, const __nv_bfloat16* bias, const uint8_t* row_mask,
                                 int zero_rows, int zero_y, const __nv_bfloat16* gamma, const __nv_bfloat16* beta,
                                 float eps, __nv_bfloat16* y, int64_t rows, int64_t D, cudaStream_t stream) {
  if (zero_rows && zero_y)
    return launch_add_layernorm_t<true, true>(resid, delta, bias, row_mask, gamma, beta, eps, y, rows, D, stream);
  if (zero_rows)
    return launch_add_layernorm_t<true, false>(resid, delta, bias, row_mask, gamma, beta, eps, y, rows, D, stream);
  if (zero_y)
    return launch_add_layernorm_t<false, true>(resid, delta, bias, row_mask, gamma, beta, eps, y, rows, D, stream);
  return launch_add_layernorm_t<false, false>(resid, delta, bias, row_mask, gamma, beta, eps, y, rows, D, stream);
}

template <bool kInBf16>
static cudaError_t launch_layernorm_t(const void* x, const __nv_bfloat16* gamma, const __nv_bfloat16* beta, float eps,
                                      __nv_bfloat16* y, float* resid_out, const uint8_t* row_mask, int64_t rows,
                                      int64_t D, cudaStream_t stream) {
  const dim3 block(kLnWarpsPerBlock * 32);
  const dim3 grid(static_cast<unsigned>((rows + kLnWarpsPerBlock - 1) / kLnWarpsPerBlock));
  const bool aligned = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (reinterpret_cast<uintptr_t>(y) % 8 == 0) &&
                       (reinterpret_cast<uintptr_t>(gamma) % 8 == 0) && (reinterpret_cast<uintptr_t>(beta) % 8 == 0) &&
                       (resid_out == nullptr || reinterpret_cast<uintptr_t>(resid_out) % 16 == 0);
#define B2_LN_CASE(NV)                                                                                   \
  case NV:                                                                                               \
    return launch_pdl(layernorm_vec_kernel<NV, kInBf16>, grid, block, 0, stream, x, gamma, beta, eps, y, resid_out, \
                      row_mask, rows);
  if (aligned && D % 128 == 0) {
    switch (D / 128) {
      B2_LN_CASE(1)
      B2_LN_CASE(2)
      B2_LN_CASE(3)
      B2_LN_CASE(4)
      B2_LN_CASE(5)
      B2_LN_CASE(6)
      B2_LN_CASE(7)
      B2_LN_CASE(8)
      B2_LN_CASE(10)
      B2_LN_CASE(12)
      B2_LN_CASE(16)
      B2_LN_CASE(24)
      B2_LN_CASE(32)
      default:
        break;
    }
  }
#undef B2_LN_CASE
  return launch_pdl(layernorm_any_kernel<kInBf16>, grid, block, 0, stream, x, gamma, beta, eps, y, resid_out, row_mask,
                    rows, D);
}

cudaError_t launch_layernorm(const void* x, int x_is_bf16, const __nv_bfloat16* gamma, const __nv_bfloat16* beta,
                             float eps, __nv_bfloat16* y, float* resid_out, const uint8_t* row_mask, int64_t rows,
                             int64_t D, cudaStream_t stream) {
  if (x_is_bf16) return launch_layernorm_t<true>(x, gamma, beta, eps, y, resid_out, row_mask, rows, D, stream);
  return launch_layernorm_t<false>(x, gamma, beta, eps, y, nullptr, row_mask, rows, D, stream);
}

// ---------------------------------------------------------------------------------------------
// Tensor-parallel all-gather fused into LayerNorm: this rank normalises its own rows (fp32 in)
// and writes the bf16 result into the same rows of every rank's LayerNorm buffer — local stores
// for its own copy, NVLink peer stores for the others, 16 bytes per lane (a lane owns 8
// consecutive columns of each 256-column group), so each GPU receives only the other ranks'
// rows. D = 256 * NG. One warp per row; masked rows are written as 0.
// ---------------------------------------------------------------------------------------------
constexpr int kGatherMaxRanks = 8;
struct GatherDst {
  __nv_bfloat16* rank_rows[kGatherMaxRanks];  // each rank's destination for row 0 of this call
};

template <int NG>
__global__ void __launch_bounds__(kLnWarpsPerBlock * 32)
    layernorm_gather_kernel(const float* __restrict__ x, const __nv_bfloat16* __restrict__ gamma,
                            const __nv_bfloat16* __restrict__ beta, float eps, GatherDst dst, int world,
                            const uint8_t* __restrict__ row_mask, int64_t rows) {
  pdl_wait_previous_grid();
  pdl_allow_next_grid();
  constexpr int D = NG * 256;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kLnWarpsPerBlock + (threadIdx.x >> 5);
  if (row < rows) {
    uint4 out[NG];
    if (row_mask != nullptr && row_mask[row] == 0) {
#pragma unroll
      for (int g = 0; g < NG; ++g) out[g] = make_uint4(0u, 0u, 0u, 0u);
    } else {
      float v[NG][8];
      const float4* xr = reinterpret_cast<const float4*>(x + row * D);
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        const float4 a = __ldg(xr + g * 64 + lane * 2);
        const float4 b = __ldg(xr + g * 64 + lane * 2 + 1);
        v[g][0] = a.x, v[g][1] = a.y, v[g][2] = a.z, v[g][3] = a.w;
        v[g][4] = b.x, v[g][5] = b.y, v[g][6] = b.z, v[g][7] = b.w;
      }
      float s = 0.f;
#pragma unroll
      for (int g = 0; g < NG; ++g)
#pragma unroll
        for (int j = 0; j < 8; ++j) s += v[g][j];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      const float mean = s * (1.0f / D);
      float q = 0.f;
#pragma unroll
      for (int g = 0; g < NG; ++g)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float d = v[g][j] - mean;
          q = fmaf(d, d, q);
        }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
      const float rstd = rsqrtf(q * (1.0f / D) + eps);
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        const uint4 graw = __ldg(reinterpret_cast<const uint4*>(gamma) + g * 32 + lane);
        const uint4 braw = __ldg(reinterpret_cast<const uint4*>(beta) + g * 32 + lane);
        const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&graw);
        const __nv_bfloat162* bh = reinterpret_cast<const __nv_bfloat162*>(&braw);
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float o0 = fmaf((v[g][2 * j] - mean) * rstd, __low2float(gh[j]), __low2float(bh[j]));
          const float o1 = fmaf((v[g][2 * j + 1] - mean) * rstd, __high2float(gh[j]), __high2float(bh[j]));
          w[j] = pack_bf16x2(o0, o1);
        }
        out[g] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    for (int r = 0; r < world; ++r) {
      uint4* yr = reinterpret_cast<uint4*>(dst.rank_rows[r] + row * D);
#pragma unroll
      for (int g = 0; g < NG; ++g) yr[g * 32 + lane] = out[g];
    }
  }
  fence_acq_rel_sys();  // peer stores ordered before the barrier that publishes them
}

bool layernorm_gather_supported(int64_t D) { return D % 256 == 0 && D / 256 >= 1 && D / 256 <= 16; }

cudaError_t launch_layernorm_gather(const float* x, const __nv_bfloat16* gamma, const __nv_bfloat16* beta, float eps,
                                    const GatherDst& dst, int world, const uint8_t* row_mask, int64_t rows, int64_t D,
                                    cudaStream_t stream) {
  const dim3 block(kLnWarpsPerBlock * 32);
  const dim3 grid(static_cast<unsigned>((rows + kLnWarpsPerBlock - 1) / kLnWarpsPerBlock));
  switch (D / 256) {
    case 1:
      return launch_pdl(layernorm_gather_kernel<1>, grid, block, 0, stream, x, gamma, beta, eps, dst, world, row_mask, rows);
    case 2:
      return launch_pdl(layernorm_gather_kernel<2>, grid, block, 0, stream, x, gamma, beta, eps, dst, world, row_mask, rows);
    case 3:
      return launch_pdl(layernorm_gather_kernel<3>, grid, block, 0, stream, x, gamma, beta, eps, dst, world, row_mask, rows);
    case 4:
      return launch_pdl(layernorm_gather_kernel<4>, grid, block, 0, stream, x, gamma, beta, eps, dst, world, row_mask, rows);
    case 8:
      return launch_pdl(layernorm_gather_kernel<8>, grid, block, 0, stream, x, gamma, beta, eps, dst, world, row_mask, rows);
    case 16:
      return launch_pdl(layernorm_gather_kernel<16>, grid, block, 0, stream, x, gamma, beta, eps, dst, world, row_mask, rows);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace b2
