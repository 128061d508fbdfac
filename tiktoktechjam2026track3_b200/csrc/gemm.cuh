// Y = A * W^T with fused epilogues, on 5th-generation tensor cores (tcgen05.mma, fp32
// accumulators in TMEM, operands staged by TMA with 128-byte swizzle).
//
// This replaces the nn.Linear calls of one Transformer block (transformer_benchmark/models.py:
// q/k/v_proj :51-53 as one packed [3D, D] projection, out_proj :76, ffn_in/ffn_out :734) and
// fuses the pointwise work that follows each of them in BaselineTransformerBlock.forward:
//   kEpiBias          out_bf16 = bf16(acc + bias)                       (packed QKV projection)
//   kEpiBiasGelu      out_bf16 = bf16(gelu_erf(bf16(acc + bias)))       (ffn_in + F.gelu, :734)
//   kEpiResidual      res_f32  = mask ? res + acc + bias : res           (out_proj, masked_fill :78-79, x + a :733)
//   kEpiResidualZero  res_f32  = mask ? res + acc + bias : 0             (ffn_out, x + f :734, masked_fill :736-737)
//   kEpiStoreF32      out_f32  = acc (+ bias when given)                 (tensor-parallel partial sums)
// A is [M, K] row-major bf16 (tokens x features), W is [N, K] row-major bf16 (nn.Linear layout,
// i.e. K-major for the B operand), the residual stream is fp32 [M, ldo].
//
// Kernel structure (one CTA per SM, persistent over 128 x BN output tiles, m-major tile order):
//   warp 0      TMA producer: A tile 128x64 and W tile BNx64 per k-block into a kStages ring.
//   warp 1      TMEM allocator and single-thread UMMA issuer (128xBNx16 per instruction);
//               tcgen05.commit frees smem stages and publishes finished accumulators.
//   warps 2..9  epilogue: tcgen05.ld of the accumulator rows owned by the warp's TMEM lane
//               quadrant (two warps per quadrant, one per half of the columns), fused pointwise
//               op, stores to global memory.
// Two TMEM accumulators (2 x BN fp32 columns) let the epilogue of tile i overlap the main loop
// of tile i+1.
#include <mutex>

#pragma once
#include "b2_common.cuh"

namespace b2 {

enum GemmEpilogue : int {
  kEpiBias = 0,
  kEpiBiasGelu = 1,
  kEpiResidual = 2,
  kEpiResidualZero = 3,
  kEpiStoreF32 = 4,
};

struct GemmParams {
  void* out;
  int64_t ldo;
  const __nv_bfloat16* bias;
  const uint8_t* row_mask;
  int M, N, K;
  int m_blocks, n_blocks, k_blocks;
};

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmThreads = 320;
constexpr int kGemmEpilogueThreads = 256;

template <int BN>
struct GemmCfg {
  static constexpr int kStages = BN == 256 ? 4 : (BN == 192 ? 5 : 6);
  static constexpr int kABytes = kGemmBM * kGemmBK * 2;
  static constexpr int kBBytes = BN * kGemmBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kAccStride = BN == 192 ? 256 : BN;  // TMEM column distance of the 2 accumulators
  static constexpr int kTmemCols = 2 * kAccStride;          // a power of two, as tcgen05.alloc requires
  static constexpr int kBarrierBytes = 256;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 + kBarrierBytes;
};

__device__ __forceinline__ void load_bias32(const __nv_bfloat16* bias, int col0, float (&b)[32]) {
  if (bias == nullptr) {
#pragma unroll
    for (int i = 0; i < 32; ++i) b[i] = 0.f;
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(bias + col0);
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    uint4 raw = __ldg(src + v);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      b[v * 8 + 2 * k] = __low2float(h[k]);
      b[v * 8 + 2 * k + 1] = __high2float(h[k]);
    }
  }
}

template <int EPI>
__device__ __forceinline__ void gemm_epilogue_chunk(const GemmParams& p, int row, int col0, const float (&acc)[32]) {
  float b[32];
  load_bias32(p.bias, col0, b);
  if constexpr (EPI == kEpiBias || EPI == kEpiBiasGelu) {
    uint32_t packed[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float x0 = acc[2 * i] + b[2 * i];
      float x1 = acc[2 * i + 1] + b[2 * i + 1];
      if constexpr (EPI == kEpiBiasGelu) {
        x0 = gelu_erf(bf16_round(x0));
        x1 = gelu_erf(bf16_round(x1));
      }
      packed[i] = pack_bf16x2(x0, x1);
    }
    uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + static_cast<int64_t>(row) * p.ldo + col0);
#pragma unroll
    for (int v = 0; v < 4; ++v)
      dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
  } else if constexpr (EPI == kEpiResidual || EPI == kEpiResidualZero) {
    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + static_cast<int64_t>(row) * p.ldo + col0);
    const bool keep = (p.row_mask == nullptr) || (p.row_mask[row] != 0);
    if (keep) {
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        float4 r = dst[v];
        r.x += acc[4 * v + 0] + b[4 * v + 0];
        r.y += acc[4 * v + 1] + b[4 * v + 1];
        r.z += acc[4 * v + 2] + b[4 * v + 2];
        r.w += acc[4 * v + 3] + b[4 * v + 3];
        dst[v] = r;
      }
    } else if constexpr (EPI == kEpiResidualZero) {
#pragma unroll
      for (int v = 0; v < 8; ++v) dst[v] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  } else {  // kEpiStoreF32
    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + static_cast<int64_t>(row) * p.ldo + col0);
#pragma unroll
    for (int v = 0; v < 8; ++v)
      dst[v] = make_float4(acc[4 * v] + b[4 * v], acc[4 * v + 1] + b[4 * v + 1], acc[4 * v + 2] + b[4 * v + 2],
                           acc[4 * v + 3] + b[4 * v + 3]);
  }
}

// Waits for a phase without looking at the abort flag (used only on the abort path, to let
// copies and MMAs that are still in flight land before the CTA releases its memory).
__device__ __forceinline__ void mbar_drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > kWaitTimeoutNs) return;
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                   const GemmParams p) {
  using Cfg = GemmCfg<BN>;
  constexpr int kStages = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_a = smem;
  uint8_t* s_b = smem + kStages * Cfg::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(s_b + kStages * Cfg::kBBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kGemmEpilogueThreads);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = p.m_blocks * p.n_blocks;

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m_blk = tile / p.n_blocks;
        const int n_blk = tile % p.n_blocks;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, kKernelGemm, 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
          tma_load_2d(s_a + s * Cfg::kABytes, &tm_a, &full[s], kb * kGemmBK, m_blk * kGemmBM);
          tma_load_2d(s_b + s * Cfg::kBBytes, &tm_b, &full[s], kb * kGemmBK, n_blk * BN);
          ++issued;
          if (++s == kStages) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let the copies still in flight (at most the last kStages issued) land before exit.
        int n = issued < kStages ? issued : kStages;
        int ss = s;
        uint32_t pp = ph;
        for (int i = 0; i < n; ++i) {
          if (--ss < 0) {
            ss = kStages - 1;
            pp ^= 1u;
          }
          mbar_drain_wait(&full[ss], pp);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16_f32(kGemmBM, BN, 0, 0);
      int s = 0;
      uint32_t ph = 0;
      int local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_ph = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_ph ^ 1u, abort_flag, kKernelGemm, 2)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * Cfg::kAccStride);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_flag, kKernelGemm, 3)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t a_addr = smem_u32(s_a + s * Cfg::kABytes);
          const uint32_t b_addr = smem_u32(s_b + s * Cfg::kBBytes);
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k) {
            const uint64_t a_desc = make_sdesc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t b_desc = make_sdesc_sw128(b_addr + k * 32, 16, 1024);
            umma_bf16_ss(d_tmem, a_desc, b_desc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[s]);
          if (++s == kStages) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);
      }
      // Every MMA this thread issued is complete once `drain` flips (normal and abort paths).
      umma_commit(drain);
      mbar_drain_wait(drain, 0);
    }
  } else {
    // Two warps per TMEM lane quadrant; each covers one half of the tile's columns.
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = quad * 32 + lane;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int m_blk = tile / p.n_blocks;
      const int n_blk = tile % p.n_blocks;
      const int acc = local & 1;
      const uint32_t acc_ph = (local >> 1) & 1;
      if (!mbar_wait(&acc_full[acc], acc_ph, abort_flag, kKernelGemm, 4)) break;
      tc_fence_after_sync();
      const int row = m_blk * kGemmBM + row_in_tile;
      const uint32_t t_row =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * Cfg::kAccStride);
#pragma unroll 1
      for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
        const int col0 = n_blk * BN + c * 32;
        if (col0 >= p.N) break;  // warp-uniform
        float v[32];
        tmem_load_32cols(t_row + c * 32, v);
        if (row < p.M) gemm_epilogue_chunk<EPI>(p, row, col0, v);
      }
      tc_fence_before_sync();
      mbar_arrive(&acc_empty[acc]);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------
cudaError_t make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                              uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer);
int device_sm_count(int device);

template <int BN, int EPI>
static cudaError_t launch_gemm_t(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int grid,
                                 cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    Cfg::kSmemBytes);
  });
  if (attr_err != cudaSuccess) return attr_err;
  gemm_tc_kernel<BN, EPI><<<grid, kGemmThreads, Cfg::kSmemBytes, stream>>>(ta, tb, p);
  return cudaGetLastError();
}

template <int BN>
static cudaError_t dispatch_epi(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int grid,
                                cudaStream_t stream) {
  switch (epi) {
    case kEpiBias:
      return launch_gemm_t<BN, kEpiBias>(ta, tb, p, grid, stream);
    case kEpiBiasGelu:
      return launch_gemm_t<BN, kEpiBiasGelu>(ta, tb, p, grid, stream);
    case kEpiResidual:
      return launch_gemm_t<BN, kEpiResidual>(ta, tb, p, grid, stream);
    case kEpiResidualZero:
      return launch_gemm_t<BN, kEpiResidualZero>(ta, tb, p, grid, stream);
    case kEpiStoreF32:
      return launch_gemm_t<BN, kEpiStoreF32>(ta, tb, p, grid, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

// Picks the N tile by the fraction of SM slots the tiles fill (waves rounded up), weighted by how
// well each tile width keeps the tensor core fed from shared memory (128x256 best). 192 exists for
// the D=768 projections: 768 = 4 x 192 gives one nearly full wave at M=4096 where 256 leaves a
// third of the SMs idle.
int gemm_pick_bn(int M, int N, int sm_count) {
  const long m_blocks = (M + kGemmBM - 1) / kGemmBM;
  const int candidates[3] = {256, 192, 128};
  const double intensity[3] = {1.0, 0.97, 0.85};
  int best = 128;
  double best_score = -1.0;
  for (int i = 0; i < 3; ++i) {
    const int bn = candidates[i];
    if (bn != 128 && N % bn != 0) continue;
    const long tiles = m_blocks * ((N + bn - 1) / bn);
    const long waves = (tiles + sm_count - 1) / sm_count;
    const double score = intensity[i] * static_cast<double>(tiles) / static_cast<double>(waves * sm_count);
    if (score > best_score + 1e-9) {
      best = bn;
      best_score = score;
    }
  }
  return best;
}

cudaError_t launch_gemm(const __nv_bfloat16* A, const __nv_bfloat16* W, const __nv_bfloat16* bias, int64_t M,
                        int64_t N, int64_t K, int epi, void* out, int64_t ldo, const uint8_t* row_mask, int bn,
                        cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = device_sm_count(dev);
  if (bn == 0) bn = gemm_pick_bn(static_cast<int>(M), static_cast<int>(N), sms);
  CUtensorMap ta, tb;
  cudaError_t e = make_tmap_bf16_2d(&ta, A, K, M, K * 2, kGemmBK, kGemmBM);
  if (e != cudaSuccess) return e;
  e = make_tmap_bf16_2d(&tb, W, K, N, K * 2, kGemmBK, bn);
  if (e != cudaSuccess) return e;
  GemmParams p;
  p.out = out;
  p.ldo = ldo;
  p.bias = bias;
  p.row_mask = row_mask;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.m_blocks = static_cast<int>((M + kGemmBM - 1) / kGemmBM);
  p.n_blocks = static_cast<int>((N + bn - 1) / bn);
  p.k_blocks = static_cast<int>((K + kGemmBK - 1) / kGemmBK);
  const long tiles = static_cast<long>(p.m_blocks) * p.n_blocks;
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);
  if (bn == 256) return dispatch_epi<256>(epi, ta, tb, p, grid, stream);
  if (bn == 192) return dispatch_epi<192>(epi, ta, tb, p, grid, stream);
  return dispatch_epi<128>(epi, ta, tb, p, grid, stream);
}

}  // namespace b2
