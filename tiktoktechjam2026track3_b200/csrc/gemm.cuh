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
//   kEpiRsResidual    owner(row).res_f32 += acc (+ bias), kept rows       (tensor parallel, fused reduce-scatter)
//   kEpiRsResidualZero  same, and masked rows set to 0 by their owner
// The two kEpiRs* epilogues add each output row into the fp32 residual of the tensor-parallel
// rank that owns the row (row / rows_per_rank) with system-scope atomics, over NVLink for the
// other ranks' rows, while the rest of the GEMM still runs; the caller passes the bias on one
// rank only and orders the owners' reads with cross-GPU barriers before and after the GEMM.
//   kEpiResidualLn      kEpiResidual, then ln_out_bf16 = LayerNorm(res_f32 row)        (out_proj + norm2)
//   kEpiResidualZeroLn  kEpiResidualZero, then ln_out_bf16 = LayerNorm(res_f32 row)    (ffn_out + next norm1)
// The two *Ln epilogues need whole rows: they run as clusters of N / BN CTAs, CTA r of a cluster
// computing column block r of the same 128 rows. Each epilogue warp reduces its rows' values to
// (mean, sum of squared deviations) pairs, merges them pairwise (Chan et al.'s update for
// combining variances), and sends them to every CTA of the cluster through distributed shared
// memory in one exchange; every CTA merges the pairs in the same fixed order, so all of them
// normalise a row with bit-identical statistics (nn.LayerNorm's biased variance). The updated
// residual waits in the TMEM accumulator during the exchange; it is read from HBM once and
// written once, after the exchange, together with the LayerNorm output.
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
#include <atomic>
#include <cstring>
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
  kEpiRsResidual = 5,
  kEpiRsResidualZero = 6,
  kEpiBiasPeers = 7,
  kEpiResidualLn = 8,
  kEpiResidualZeroLn = 9,
};

constexpr int kGemmMaxPeers = 8;

struct GemmParams {
  void* out;
  int64_t ldo;
  const __nv_bfloat16* bias;
  const uint8_t* row_mask;
  int M, N, K;
  int m_blocks, n_blocks, k_blocks;
  // kEpiRs*: every rank's residual base (as mapped here); row r belongs to rank r / rows_per_rank.
  // kEpiBiasPeers: every rank's output base; columns >= peer_col go to every rank's copy.
  void* peer_out[kGemmMaxPeers];
  int rows_per_rank, world, rank, peer_col;
  // kEpi*Ln: LayerNorm of the updated residual rows into ln_out [M, N] bf16 (row stride N).
  const __nv_bfloat16* ln_gamma;
  const __nv_bfloat16* ln_beta;
  __nv_bfloat16* ln_out;
  float ln_eps;
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

template <int EPI>
__host__ __device__ constexpr bool is_rs_epi() {
  return EPI == kEpiRsResidual || EPI == kEpiRsResidualZero;
}
template <int EPI>
__host__ __device__ constexpr bool is_ln_epi() {
  return EPI == kEpiResidualLn || EPI == kEpiResidualZeroLn;
}

// Row-statistics exchange of the *Ln epilogues: 8 mbarriers [tile parity][TMEM lane quadrant] and
// the (mean, M2) pairs [tile parity][quadrant][source = 2 * cluster rank + column half][32 rows].
// Senders write with st.async, which counts the bytes on the receiver's barrier; each barrier is
// armed (expect_tx of all 2 * cs * 256 bytes) before any sender can write its phase: at launch
// for the first two tiles, and by the receiver right after it has read a phase's pairs for the
// phase two tiles later. No CTA gets two tiles ahead of another (that needs the slow CTA's pairs),
// so the two parities keep tile t+1's pairs off the slots and the barrier of tile t.
constexpr int kLnMaxCluster = 8;
constexpr int kLnBarrierBytes = 128;
constexpr int kLnBytes = kLnBarrierBytes + 2 * 4 * (2 * kLnMaxCluster) * 32 * 8;

// Epilogue staging: TMEM gives each lane one row of the accumulator, so a lane writing its own
// row would make every warp-wide global access touch 32 different rows (32 memory transactions
// of 16 bytes per instruction, and for the reduce-scatter epilogues 32 NVLink requests). Each epilogue
// warp therefore passes its 32 x 32 fp32 chunk through 4 KB of shared memory and then works on
// whole row segments: lane i handles columns 4(i % 8) .. +3 of rows i / 8, 4 + i / 8, ...
constexpr int kEpiStageBytes = (kGemmThreads / 32 - 2) * 32 * 32 * 4;

template <int BN, int EPI>
struct GemmSmem {
  static constexpr int kFixed =
      1024 + GemmCfg<BN>::kBarrierBytes + kEpiStageBytes + (is_ln_epi<EPI>() ? kLnBytes : 0);
  static constexpr int kWant = BN == 192 ? 4 : GemmCfg<BN>::kStages;
  static constexpr int kFit = (232448 - kFixed) / GemmCfg<BN>::kStageBytes;
  static constexpr int kStages = kWant < kFit ? kWant : kFit;
  static constexpr int kBytes = kStages * GemmCfg<BN>::kStageBytes + kFixed;
  static_assert(kStages >= 3 && kBytes <= 232448, "shared memory per CTA");
};

__device__ __forceinline__ float4 load_bias4(const __nv_bfloat16* bias, int col) {
  if (bias == nullptr) return make_float4(0.f, 0.f, 0.f, 0.f);
  const uint2 raw = __ldg(reinterpret_cast<const uint2*>(bias + col));
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
  return make_float4(__low2float(h[0]), __high2float(h[0]), __low2float(h[1]), __high2float(h[1]));
}

// Row flags of the 8 rows a lane serves in the transposed layout below (rows row0 + 4i + lane / 8):
// bit i of live = the row is inside M, of keep = inside M and kept by the row mask. Computed once
// per tile (the row mask bytes are then not re-read for every chunk).
__device__ __forceinline__ void gemm_epi_row_bits(const GemmParams& p, int row0, uint32_t& live, uint32_t& keep) {
  const int lane = threadIdx.x & 31;
  live = 0;
  keep = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int row = row0 + i * 4 + (lane >> 3);
    if (row < p.M) {
      live |= 1u << i;
      if (p.row_mask == nullptr || p.row_mask[row] != 0) keep |= 1u << i;
    }
  }
}

template <int EPI>
__host__ __device__ constexpr bool epi_reads_residual() {
  return EPI == kEpiResidual || EPI == kEpiResidualZero;
}

// TMEM gives each lane one row of the accumulator, so a lane writing its own row would make every
// warp-wide global access touch 32 different rows. The warp therefore passes its 32 x 32 fp32 chunk
// through 4 KB of shared memory: row `lane` as 8 float4 pieces, the piece index XOR-swizzled by the
// row, so that both these stores (8 lanes = 8 rows, same piece) and the loads in
// gemm_epilogue_chunk (8 lanes = one row, 8 pieces) spread over all 32 banks.
__device__ __forceinline__ void gemm_epi_stage(const float (&acc)[32], float4* stage) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int c = 0; c < 8; ++c)
    stage[lane * 8 + (c ^ (lane & 7))] = make_float4(acc[4 * c], acc[4 * c + 1], acc[4 * c + 2], acc[4 * c + 3]);
  __syncwarp();
}

// One warp's 32 rows x 32 columns after gemm_epi_stage (row0 = the warp's first row): lane i
// handles columns 4(i % 8) .. +3 of rows i / 8, 4 + i / 8, ... (v[j] = row 4j + i / 8), reading them
// back from the staging buffer with the bias added.
__device__ __forceinline__ void gemm_epi_gather(const float4* stage, const float4& b, float4 (&v)[8]) {
  const int lane = threadIdx.x & 31;
  const int q = lane & 7;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = i * 4 + (lane >> 3);
    v[i] = stage[r * 8 + (q ^ (r & 7))];
    v[i].x += b.x;
    v[i].y += b.y;
    v[i].z += b.z;
    v[i].w += b.w;
  }
}

// Writes one gathered chunk (for the residual epilogues v already holds residual + acc + bias on
// kept rows). Rows >= M are skipped.
template <int EPI>
__device__ __forceinline__ void gemm_epi_store(const GemmParams& p, int row0, int col0, const float4 (&v)[8],
                                               uint32_t live, uint32_t keep) {
  const int lane = threadIdx.x & 31;
  const int col = col0 + 4 * (lane & 7);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (!((live >> i) & 1u)) continue;
    const int64_t off = static_cast<int64_t>(row0 + i * 4 + (lane >> 3)) * p.ldo + col;
    if constexpr (epi_reads_residual<EPI>()) {
      float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + off);
      if ((keep >> i) & 1u)
        *dst = v[i];
      else if (EPI == kEpiResidualZero)
        *dst = make_float4(0.f, 0.f, 0.f, 0.f);
    } else if constexpr (EPI == kEpiBias || EPI == kEpiBiasGelu || EPI == kEpiBiasPeers) {
      float4 w = v[i];
      if constexpr (EPI == kEpiBiasGelu) {
        w.x = gelu_erf(bf16_round(w.x));
        w.y = gelu_erf(bf16_round(w.y));
        w.z = gelu_erf(bf16_round(w.z));
        w.w = gelu_erf(bf16_round(w.w));
      }
      const uint2 packed = make_uint2(pack_bf16x2(w.x, w.y), pack_bf16x2(w.z, w.w));
      *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.out) + off) = packed;
      if constexpr (EPI == kEpiBiasPeers) {
        if (col0 >= p.peer_col) {  // warp-uniform: a chunk's 32 columns are on one side
          for (int r = 0; r < p.world; ++r)
            if (r != p.rank) *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.peer_out[r]) + off) = packed;
        }
      }
    } else if constexpr (EPI == kEpiStoreF32) {
      *reinterpret_cast<float4*>(static_cast<float*>(p.out) + off) = v[i];
    } else {  // reduce-scatter: the row owner's copy
      const int row = row0 + i * 4 + (lane >> 3);
      const int owner = min(row / p.rows_per_rank, p.world - 1);
      float* dst = static_cast<float*>(p.peer_out[owner]) + off;
      if ((keep >> i) & 1u)
        red_add_v4_sys(dst, v[i].x, v[i].y, v[i].z, v[i].w);
      else if (EPI == kEpiRsResidualZero && owner == p.rank)
        *reinterpret_cast<float4*>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
}

// The operands of one warp's epilogue that do not depend on the accumulator: the row flags, the
// bias of every chunk of the warp's columns and, for the residual epilogues, the residual rows of
// its first chunk. They are loaded before the warp waits for the accumulator, so their latency
// (a DRAM round trip for the bias right after the weights change, an L2 one otherwise) hides
// behind the main loop instead of stalling each chunk. A per-CTA trace of C2's GEMMs
// (%globaltimer stamps; 128 x 256 GELU tile) had the epilogue at 8.6 us against a 4.6 us main loop
// while each chunk waited for its bias load and its TMEM load in turn.
template <int BN, int EPI>
struct EpiPrefetch {
  uint32_t live, keep;
  float4 bias[BN / 64];
  float4 res[8];
};

template <int EPI>
__device__ __forceinline__ void gemm_epi_fetch_residual(const GemmParams& p, int row0, int col0, uint32_t keep,
                                                        float4 (&res)[8]) {
  const int lane = threadIdx.x & 31;
  const int col = col0 + 4 * (lane & 7);
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if ((keep >> i) & 1u)
      res[i] = *reinterpret_cast<const float4*>(static_cast<const float*>(p.out) +
                                                static_cast<int64_t>(row0 + i * 4 + (lane >> 3)) * p.ldo + col);
}

template <int BN, int EPI>
__device__ __forceinline__ void gemm_epi_prefetch(const GemmParams& p, int row0, int n_blk, int half,
                                                  EpiPrefetch<BN, EPI>& pre) {
  gemm_epi_row_bits(p, row0, pre.live, pre.keep);
  const int lane = threadIdx.x & 31;
  const int c_begin = half * (BN / 64);
#pragma unroll
  for (int c = 0; c < BN / 64; ++c) {
    const int col0 = n_blk * BN + (c_begin + c) * 32;
    pre.bias[c] = col0 < p.N ? load_bias4(p.bias, col0 + 4 * (lane & 7)) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if constexpr (epi_reads_residual<EPI>()) {
    if (n_blk * BN + c_begin * 32 < p.N) gemm_epi_fetch_residual<EPI>(p, row0, n_blk * BN + c_begin * 32, pre.keep,
                                                                      pre.res);
  }
}

// The bf16-output epilogues (bias, bias + GELU, bias + peer stores) of one tile for one warp. The
// pointwise work runs in the TMEM layout (lane = row, 32 consecutive columns per chunk), the bias
// read from shared memory as broadcasts, and only the bf16 results pass through the staging
// buffer on their way to coalesced 16-byte row segments: half the shared-memory bytes of staging
// the fp32 accumulator, which the tcgen05.mma of the next tile competes with for bandwidth (the
// main loop ran ~1.4x slower under the fp32-staged epilogue in a per-CTA trace).
// Staging layout per warp (4 KB): [0, 2 KB) the chunk's 32 rows x 64 B, 16-byte pieces XOR-swizzled
// by (row / 2) % 4, so that both the row-wise stores and the transposed loads hit 32 distinct
// banks per quarter-warp; [2 KB, +BN/2 x 4 B) the bias of the warp's columns.
template <int BN, int EPI>
__device__ __forceinline__ void gemm_epilogue_tile_bf16(const GemmParams& p, int row0, int n_blk, int half,
                                                        uint32_t t_row, float4* stage, EpiPrefetch<BN, EPI>& pre) {
  constexpr int kC = BN / 64;
  const int lane = threadIdx.x & 31;
  const int c_begin = half * kC;
  int n_valid = 0;
#pragma unroll
  for (int c = 0; c < kC; ++c)
    if (n_blk * BN + (c_begin + c) * 32 < p.N) n_valid = c + 1;
  if (n_valid == 0) return;
  uint4* rows = reinterpret_cast<uint4*>(stage);
  float4* bias_s = stage + 128;
  if (lane < 8) {
#pragma unroll
    for (int c = 0; c < kC; ++c) bias_s[c * 8 + lane] = pre.bias[c];
  }
  uint32_t buf[2][32];
  tmem_ld32_issue(t_row + c_begin * 32, buf[0]);
  __syncwarp();
#pragma unroll
  for (int c = 0; c < kC; ++c) {
    if (c >= n_valid) break;
    uint32_t(&cur)[32] = buf[c & 1];
    tmem_ld32_wait(cur);
    if (c + 1 < n_valid) tmem_ld32_issue(t_row + (c_begin + c + 1) * 32, buf[(c + 1) & 1]);
    uint32_t pk[16];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 b = bias_s[c * 8 + j];
      float x0 = __uint_as_float(cur[4 * j]) + b.x, x1 = __uint_as_float(cur[4 * j + 1]) + b.y;
      float x2 = __uint_as_float(cur[4 * j + 2]) + b.z, x3 = __uint_as_float(cur[4 * j + 3]) + b.w;
      if constexpr (EPI == kEpiBiasGelu) {
        x0 = bf16_round(x0);
        x1 = bf16_round(x1);
        x2 = bf16_round(x2);
        x3 = bf16_round(x3);
        gelu_erf2(x0, x1);
        gelu_erf2(x2, x3);
      }
      pk[2 * j] = pack_bf16x2(x0, x1);
      pk[2 * j + 1] = pack_bf16x2(x2, x3);
    }
    const int sw = (lane >> 1) & 3;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      rows[lane * 4 + (q ^ sw)] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
    __syncwarp();
    const int col0 = n_blk * BN + (c_begin + c) * 32;
    const int piece = lane & 3;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = 8 * i + (lane >> 2);
      const uint4 v = rows[r * 4 + (piece ^ ((r >> 1) & 3))];
      const int row = row0 + r;
      if (row < p.M) {
        const int64_t off = static_cast<int64_t>(row) * p.ldo + col0 + 8 * piece;
        *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + off) = v;
        if constexpr (EPI == kEpiBiasPeers) {
          if (col0 >= p.peer_col) {  // warp-uniform: a chunk's 32 columns are on one side
            for (int rk = 0; rk < p.world; ++rk)
              if (rk != p.rank) *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.peer_out[rk]) + off) = v;
          }
        }
      }
    }
    __syncwarp();  // the staging rows are rewritten by the next chunk
  }
}

// The epilogue of one tile for one warp: its TMEM lane quadrant (t_row) and its half of the tile's
// columns, in 32-column chunks, with the operands `pre` loaded before the accumulator was ready.
// The next chunk's TMEM load is issued before the current chunk is processed (two register
// buffers), and the residual epilogues fetch the next chunk's residual rows as soon as the current
// ones are consumed, so each chunk's latencies overlap the previous chunk's work.
template <int BN, int EPI>
__device__ __forceinline__ void gemm_epilogue_tile(const GemmParams& p, int row0, int n_blk, int half, uint32_t t_row,
                                                   float4* stage, EpiPrefetch<BN, EPI>& pre) {
  if constexpr (EPI == kEpiBias || EPI == kEpiBiasGelu || EPI == kEpiBiasPeers) {
    gemm_epilogue_tile_bf16<BN, EPI>(p, row0, n_blk, half, t_row, stage, pre);
    return;
  }
  constexpr int kC = BN / 64;
  const int c_begin = half * kC;
  int n_valid = 0;  // chunks inside N (a prefix; warp-uniform)
#pragma unroll
  for (int c = 0; c < kC; ++c)
    if (n_blk * BN + (c_begin + c) * 32 < p.N) n_valid = c + 1;
  if (n_valid == 0) return;
  // The residual epilogues hold a chunk of residual rows in registers as well: there each TMEM
  // load is waited for at once (a second buffer made ptxas spill, and no register that a pending
  // tcgen05.ld writes may be spilled), the others keep two buffers.
  constexpr int kBufs = epi_reads_residual<EPI>() ? 1 : 2;
  uint32_t buf[kBufs][32];
  if (kBufs == 2) tmem_ld32_issue(t_row + c_begin * 32, buf[0]);
#pragma unroll
  for (int c = 0; c < kC; ++c) {
    if (c >= n_valid) break;
    uint32_t(&cur)[32] = buf[c % kBufs];
    if (kBufs == 1) tmem_ld32_issue(t_row + (c_begin + c) * 32, cur);
    tmem_ld32_wait(cur);
    if (kBufs == 2 && c + 1 < n_valid) tmem_ld32_issue(t_row + (c_begin + c + 1) * 32, buf[(c + 1) % kBufs]);
    const int col0 = n_blk * BN + (c_begin + c) * 32;
    {
      float acc[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[i] = __uint_as_float(cur[i]);
      gemm_epi_stage(acc, stage);
    }
    float4 v[8];
    gemm_epi_gather(stage, pre.bias[c], v);
    if constexpr (epi_reads_residual<EPI>()) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if ((pre.keep >> i) & 1u)
          v[i] = make_float4(pre.res[i].x + v[i].x, pre.res[i].y + v[i].y, pre.res[i].z + v[i].z,
                             pre.res[i].w + v[i].w);
      if (c + 1 < n_valid) gemm_epi_fetch_residual<EPI>(p, row0, col0 + 32, pre.keep, pre.res);
    }
    gemm_epi_store<EPI>(p, row0, col0, v, pre.live, pre.keep);
    __syncwarp();  // the staging buffer is rewritten by the next chunk
  }
}

// Pass 1 of the *Ln epilogues for one warp's 32 rows x 32 columns (layout as in
// gemm_epilogue_chunk): the updated residual values come back in `vals` (lane i: rows 4j + i / 8,
// columns 4(i % 8) .. +3, j = 0..7, as vals[4j .. 4j+3]); nothing is stored yet. Per row j the
// lane accumulates sum[j] and sq[j] = sum of (x - shift[j])^2, shift[j] being its first value of
// the row (so the variance does not cancel when the mean is large). Bit j of keep_bits / live_bits:
// the row is kept by the mask / inside M. Masked rows keep their residual (kEpiResidualLn) or
// become 0 (kEpiResidualZeroLn); either way they are normalised like the others, as nn.LayerNorm does.
template <int EPI>
__device__ __forceinline__ void gemm_ln_chunk(const GemmParams& p, int row0, int col0, float (&vals)[32],
                                              float4* stage, bool first, float (&sum)[8], float (&sq)[8],
                                              float (&shift)[8], uint32_t& keep_bits, uint32_t& live_bits) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int c = 0; c < 8; ++c)
    stage[lane * 8 + (c ^ (lane & 7))] = make_float4(vals[4 * c], vals[4 * c + 1], vals[4 * c + 2], vals[4 * c + 3]);
  __syncwarp();
  const int q = lane & 7;
  const int col = col0 + 4 * q;
  const float4 b = load_bias4(p.bias, col);
  float4 v[8], res[8];
  bool live[8], keep[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = i * 4 + (lane >> 3);
    const int row = row0 + r;
    v[i] = stage[r * 8 + (q ^ (r & 7))];
    live[i] = row < p.M;
    keep[i] = live[i] && (p.row_mask == nullptr || p.row_mask[row] != 0);
    res[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t off = static_cast<int64_t>(row0 + i * 4 + (lane >> 3)) * p.ldo + col;
    const bool need = EPI == kEpiResidualLn ? live[i] : keep[i];
    if (need) res[i] = *reinterpret_cast<const float4*>(static_cast<const float*>(p.out) + off);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float4 o = res[i];
    if (keep[i]) {
      o.x += v[i].x + b.x;
      o.y += v[i].y + b.y;
      o.z += v[i].z + b.z;
      o.w += v[i].w + b.w;
    }
    keep_bits |= keep[i] ? (1u << i) : 0u;
    live_bits |= live[i] ? (1u << i) : 0u;
    vals[4 * i] = o.x;
    vals[4 * i + 1] = o.y;
    vals[4 * i + 2] = o.z;
    vals[4 * i + 3] = o.w;
    if (first) shift[i] = o.x;
    sum[i] += (o.x + o.y) + (o.z + o.w);
    const float dx = o.x - shift[i], dy = o.y - shift[i], dz = o.z - shift[i], dw = o.w - shift[i];
    sq[i] = fmaf(dw, dw, fmaf(dz, dz, fmaf(dy, dy, fmaf(dx, dx, sq[i]))));
  }
  __syncwarp();
}

// Turns this lane's per-row (sum, sq, shift) over n_lane values into the row's (mean, M2) over
// the warp's columns, merged across the 8 lanes of each row (equal counts; the merge is symmetric
// in its operands, so every lane of a row ends with the same bits), sends row `lane`'s pair to
// every CTA of the cluster, waits for the cluster's pairs and merges all 2 * cs of them in source
// order into mean[j] and rstd[j] for the lane's rows 4j + lane / 8. Returns false when the wait
// gave up (status recorded, *abort raised).
__device__ __forceinline__ bool gemm_ln_stats(const GemmParams& p, int bn, float n_lane, const float (&sum)[8],
                                              const float (&sq)[8], const float (&shift)[8], float (&mean)[8],
                                              float (&rstd)[8], int quad, int half, uint32_t parity,
                                              uint32_t use_parity, uint32_t my_rank, uint64_t* xbar, float* xch,
                                              volatile int* abort) {
  const int lane = threadIdx.x & 31;
  const int cs = p.n_blocks;
  float m2[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (n_lane > 0.f) {
      mean[j] = sum[j] / n_lane;
      const float d = mean[j] - shift[j];
      m2[j] = fmaxf(sq[j] - n_lane * d * d, 0.f);
    } else {
      mean[j] = 0.f;
      m2[j] = 0.f;
    }
  }
  float n = n_lane;
#pragma unroll
  for (int o = 1; o <= 4; o <<= 1) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float mb = __shfl_xor_sync(0xffffffffu, mean[j], o);
      const float qb = __shfl_xor_sync(0xffffffffu, m2[j], o);
      const float d = mb - mean[j];
      m2[j] = (m2[j] + qb) + d * d * (0.5f * n);
      mean[j] = (mean[j] + mb) * 0.5f;
    }
    n *= 2.f;
  }
  // Lane L takes row L: row 4j + g is held by the lanes 8g .. 8g+7, j = L / 4, g = L % 4.
  float my_mean = 0.f, my_m2 = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float tm = __shfl_sync(0xffffffffu, mean[j], (lane & 3) << 3);
    const float tq = __shfl_sync(0xffffffffu, m2[j], (lane & 3) << 3);
    if ((lane >> 2) == j) {
      my_mean = tm;
      my_m2 = tq;
    }
  }
  float* block = xch + ((parity * 4 + quad) * (2 * kLnMaxCluster)) * 32 * 2;
  const uint32_t slot = smem_u32(block + ((2 * static_cast<int>(my_rank) + half) * 32 + lane) * 2);
  uint64_t* bar = &xbar[parity * 4 + quad];
  for (int r = 0; r < cs; ++r) {
    uint32_t dst, dbar;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(dst) : "r"(slot), "r"(r));
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(dbar) : "r"(smem_u32(bar)), "r"(r));
    st_async_v2f32(dst, my_mean, my_m2, dbar);
  }
  // One lane polls (test_wait: no suspension), the warp then re-converges and reads: with all 32
  // lanes in a suspending try_wait, lanes woke up microseconds after the bytes had landed.
  bool ok = true;
  if (lane == 0 && !mbar_test_wait_cluster(bar, use_parity)) {
    const uint64_t t0 = global_timer_ns();
    uint32_t spins = 0;
    while (!mbar_test_wait_cluster(bar, use_parity)) {
      if ((++spins & 63u) == 0) {
        if (*abort) {
          ok = false;
          break;
        }
        if (global_timer_ns() - t0 > wait_limit_ns()) {
          record_status(kKernelGemm, 6, kReasonTimeout);
          *abort = 1;
          ok = false;
          break;
        }
      }
    }
  }
  if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) return false;
  // Sources outer, the lane's 8 rows inner: 8 independent accumulation chains per step. Every
  // source holds bn / 2 columns except, in a single-CTA row (n <= 256), a half past n.
  const float inv_n = 1.0f / static_cast<float>(p.N);
  const float2* pairs = reinterpret_cast<const float2*>(block) + (lane >> 3);
  const int n_src = cs == 1 ? (p.N > bn / 2 ? 2 : 1) : 2 * cs;
  const float w_last = static_cast<float>(cs == 1 ? p.N - (n_src - 1) * (bn / 2) : bn / 2);
  const float w_full = static_cast<float>(bn / 2);
  float tot[8], m2t[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    tot[j] = 0.f;
    m2t[j] = 0.f;
  }
  for (int src = 0; src < n_src; ++src) {
    const float w = src == n_src - 1 ? w_last : w_full;
#pragma unroll
    for (int j = 0; j < 8; ++j) tot[j] = fmaf(w, pairs[src * 32 + j * 4].x, tot[j]);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) mean[j] = tot[j] * inv_n;
  for (int src = 0; src < n_src; ++src) {
    const float w = src == n_src - 1 ? w_last : w_full;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float2 pr = pairs[src * 32 + j * 4];
      const float d = pr.x - mean[j];
      m2t[j] += pr.y + w * d * d;
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) rstd[j] = rsqrtf(m2t[j] * inv_n + p.ln_eps);
  // Re-arm this barrier for its next phase (tile t+2). Both warps of the quadrant have seen this
  // phase complete or will (the next one needs their own bytes); the pairs just read cannot be
  // overwritten before then (a sender must first receive this CTA's pairs of tile t+1).
  __syncwarp();
  if (half == 0 && lane == 0) mbar_arrive_expect_tx(bar, static_cast<uint32_t>(2 * cs * 32 * 8));
  return true;
}

// Waits for a phase without looking at the abort flag (used only on the abort path, to let
// copies and MMAs that are still in flight land before the CTA releases its memory).
__device__ __forceinline__ void mbar_drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = global_timer_ns();
  const uint64_t lim = wait_limit_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > lim) return;
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                   const GemmParams p) {
  using Cfg = GemmCfg<BN>;
  constexpr int kStages = GemmSmem<BN, EPI>::kStages;
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
    if constexpr (is_ln_epi<EPI>()) {
      uint64_t* xbar = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(full) + Cfg::kBarrierBytes +
                                                   kEpiStageBytes);
      // One local arrival per phase (the arming expect_tx); the bytes of all 2 * cs source warps
      // complete it. Both parities are armed here, before the cluster barrier lets anyone send.
      for (int i = 0; i < 8; ++i) {
        mbar_init(&xbar[i], 1);
        mbar_arrive_expect_tx(&xbar[i], static_cast<uint32_t>(2 * p.n_blocks * 32 * 8));
      }
    }
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
  if constexpr (is_ln_epi<EPI>())
    cluster_sync_all();  // every CTA's exchange barriers exist before any remote arrive
  else
    __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = p.m_blocks * p.n_blocks;
  // The weights (B operand) do not depend on the previous kernel: the first ring's worth of W
  // tiles is requested before waiting for it (programmatic dependent launch), so their DRAM
  // latency overlaps the previous kernel's tail. A per-CTA trace showed the first stage landing
  // ~2 us after the wait when both operands were requested only then.
  int w_early = 0;
  // Test-only (b2_test_set_fault): CTA 0 leaves its first stage unarmed and unloaded.
  const bool withhold = warp == 0 && lane == 0 && blockIdx.x == 0 &&
                        *reinterpret_cast<volatile uint32_t*>(&g_test_fault) == kFaultGemmWithholdStage;
  if (warp == 0 && lane == 0) {
    for (int tile = blockIdx.x; tile < num_tiles && w_early < kStages; tile += gridDim.x) {
      const int n_blk = tile % p.n_blocks;
      for (int kb = 0; kb < p.k_blocks && w_early < kStages; ++kb, ++w_early) {
        if (withhold && w_early == 0) continue;
        mbar_arrive_expect_tx(&full[w_early], Cfg::kStageBytes);
        tma_load_2d(s_b + w_early * Cfg::kBBytes, &tm_b, &full[w_early], kb * kGemmBK, n_blk * BN);
      }
    }
  }
  pdl_wait_previous_grid();
  pdl_allow_next_grid();

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
          if (issued >= w_early) {
            mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
            tma_load_2d(s_b + s * Cfg::kBBytes, &tm_b, &full[s], kb * kGemmBK, n_blk * BN);
          }
          if (!(withhold && issued == 0))
            tma_load_2d(s_a + s * Cfg::kABytes, &tm_a, &full[s], kb * kGemmBK, m_blk * kGemmBM);
          ++issued;
          if (++s == kStages) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {
        // W tiles requested early for stages whose A tile was never issued: their barrier phase
        // cannot complete, so give those copies a fixed time to land in shared memory.
        if (w_early > issued) {
          const uint64_t t0 = global_timer_ns();
          while (global_timer_ns() - t0 < 200000ull) {
          }
        }
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
    float4* epi_stage = reinterpret_cast<float4*>(reinterpret_cast<uint8_t*>(full) + Cfg::kBarrierBytes) + (warp - 2) * 256;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int m_blk = tile / p.n_blocks;
      const int n_blk = tile % p.n_blocks;
      const int acc = local & 1;
      const uint32_t acc_ph = (local >> 1) & 1;
      const int row = m_blk * kGemmBM + row_in_tile;
      EpiPrefetch<BN, EPI> pre;
      if constexpr (!is_ln_epi<EPI>()) gemm_epi_prefetch<BN, EPI>(p, row - lane, n_blk, half, pre);
      if (!mbar_wait(&acc_full[acc], acc_ph, abort_flag, kKernelGemm, 4)) break;
      tc_fence_after_sync();
      const uint32_t t_row =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * Cfg::kAccStride);
      if constexpr (is_ln_epi<EPI>()) {
        constexpr int kChunks = BN / 64;  // 32-column chunks per warp (one half of the tile)
        uint64_t* xbar = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(full) + Cfg::kBarrierBytes +
                                                     kEpiStageBytes);
        float* xch = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xbar) + kLnBarrierBytes);
        const uint32_t my_rank = static_cast<uint32_t>(n_blk);  // == %cluster_ctarank
        const int c_first = half * kChunks;
        // gamma / beta of this lane's columns, loaded before the main work hides their latency.
        float4 g[kChunks], bt[kChunks];
#pragma unroll
        for (int c = 0; c < kChunks; ++c) {
          const int col = n_blk * BN + (c_first + c) * 32 + 4 * (lane & 7);
          g[c] = col < p.N ? load_bias4(p.ln_gamma, col) : make_float4(0.f, 0.f, 0.f, 0.f);
          bt[c] = col < p.N ? load_bias4(p.ln_beta, col) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        // Pass 1: residual update into TMEM (over the consumed accumulator), row statistics.
        float sum[8], sq[8], shift[8], mean[8], rstd[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          sum[j] = 0.f;
          sq[j] = 0.f;
          shift[j] = 0.f;
        }
        uint32_t keep_bits = 0, live_bits = 0;
        int chunks = 0;
#pragma unroll 1
        for (int c = c_first; c < c_first + kChunks; ++c) {
          const int col0 = n_blk * BN + c * 32;
          if (col0 >= p.N) break;  // warp-uniform
          float v[32];
          tmem_load_32cols(t_row + c * 32, v);
          gemm_ln_chunk<EPI>(p, row - lane, col0, v, epi_stage, c == c_first, sum, sq, shift, keep_bits, live_bits);
          tmem_store_32cols_async(t_row + c * 32, v);
          ++chunks;
        }
        tmem_wait_st();
        if (!gemm_ln_stats(p, BN, 4.0f * static_cast<float>(chunks), sum, sq, shift, mean, rstd, quad, half,
                           static_cast<uint32_t>(local & 1), static_cast<uint32_t>((local >> 1) & 1), my_rank, xbar,
                           xch, abort_flag))
          break;
        // Pass 3: store the residual (kept rows; masked rows too when they become 0) and the
        // LayerNorm output, y = (x - mean) * rstd * gamma + beta, as 8-lane row segments. Two
        // chunks per TMEM load where both exist (one load latency instead of two).
        auto finish_chunk = [&](int c, const float* v) {
          const int col = n_blk * BN + (c_first + c) * 32 + 4 * (lane & 7);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (!((live_bits >> j) & 1u)) continue;
            const int64_t r = row - lane + j * 4 + (lane >> 3);
            if (((keep_bits >> j) & 1u) || EPI == kEpiResidualZeroLn)
              *reinterpret_cast<float4*>(static_cast<float*>(p.out) + r * p.ldo + col) =
                  make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            const float y0 = fmaf((v[4 * j] - mean[j]) * rstd[j], g[c].x, bt[c].x);
            const float y1 = fmaf((v[4 * j + 1] - mean[j]) * rstd[j], g[c].y, bt[c].y);
            const float y2 = fmaf((v[4 * j + 2] - mean[j]) * rstd[j], g[c].z, bt[c].z);
            const float y3 = fmaf((v[4 * j + 3] - mean[j]) * rstd[j], g[c].w, bt[c].w);
            *reinterpret_cast<uint2*>(p.ln_out + r * p.N + col) = make_uint2(pack_bf16x2(y0, y1), pack_bf16x2(y2, y3));
          }
        };
#pragma unroll
        for (int c = 0; c < kChunks; c += 2) {
          const int col0 = n_blk * BN + (c_first + c) * 32;
          if (col0 >= p.N) break;  // warp-uniform
          if (c + 1 < kChunks && col0 + 32 < p.N) {
            float v[64];
            tmem_load_64cols(t_row + (c_first + c) * 32, v);
            finish_chunk(c, v);
            finish_chunk(c + 1, v + 32);
          } else {
            float v[32];
            tmem_load_32cols(t_row + (c_first + c) * 32, v);
            finish_chunk(c, v);
          }
        }
      } else {
        gemm_epilogue_tile<BN, EPI>(p, row - lane, n_blk, half, t_row, epi_stage, pre);
      }
      tc_fence_before_sync();
      mbar_arrive(&acc_empty[acc]);
    }
    if constexpr (is_rs_epi<EPI>() || EPI == kEpiBiasPeers) fence_acq_rel_sys();
  }

  if (is_ln_epi<EPI>() && *abort_flag && threadIdx.x == 0) {
    // A wait gave up: give row-statistics stores still in flight to or from this CTA time to land.
    const uint64_t t0 = global_timer_ns();
    while (global_timer_ns() - t0 < 200000ull) {
    }
  }
  __syncthreads();
  if constexpr (is_ln_epi<EPI>()) cluster_sync_all();  // no CTA leaves while others may still write to it
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------
// 2-SM variant: a cluster of 2 CTAs computes a 256 x BN tile with tcgen05.mma.cta_group::2. CTA
// p of the pair loads A rows [128p, 128p + 128) and W rows [BN/2 p, BN/2 (p+1)) of the tile
// (32 KB per 64-deep k-block for BN = 256, against 48 KB per CTA for a 128 x 256 one-CTA tile), so
// every byte fetched from L2 feeds 1.5x more MMA work, and the 32 KB stages allow a 6-deep ring.
// The leader (rank 0) issues the MMAs; both CTAs' TMA loads count on the leader's full barrier;
// the leader's commits reach both CTAs' empty / accumulator barriers; each CTA's epilogue drains
// its own 128 accumulator rows and reports to the leader's acc_empty barrier.
// ---------------------------------------------------------------------------------------------
template <int BN>
struct Gemm2Cfg {
  static constexpr int kStages = 6;
  static constexpr int kABytes = 128 * kGemmBK * 2;             // this CTA's 128 rows of A
  static constexpr int kBBytes = (BN / 2) * kGemmBK * 2;        // this CTA's BN/2 rows of W
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kAccStride = 256;
  static constexpr int kTmemCols = 512;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256;
};
template <int BN, int EPI>
constexpr int gemm2_smem_bytes() {
  return Gemm2Cfg<BN>::kSmemBytes + kEpiStageBytes;
}

template <int BN, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    const GemmParams p) {
  using Cfg = Gemm2Cfg<BN>;
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
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(cluster_id_x());
  const int n_pairs = static_cast<int>(cluster_count_x());

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * kGemmEpilogueThreads);
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
    tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before_sync();
  cluster_sync_all();  // both CTAs' barriers exist before any remote arrive / transaction
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait_previous_grid();
  pdl_allow_next_grid();

  const int m_tiles = (p.M + 255) / 256;
  const int num_tiles = m_tiles * p.n_blocks;

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += n_pairs) {
        const int m_blk = tile / p.n_blocks;
        const int n_blk = tile % p.n_blocks;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, kKernelGemm, 11)) {
            ok = false;
            break;
          }
          const uint32_t bar = cluster_map_to_rank(&full[s], 0);
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * Cfg::kStageBytes);
          tma_load_2d_pair(s_a + s * Cfg::kABytes, &tm_a, bar, kb * kGemmBK, m_blk * 256 + rank * 128);
          tma_load_2d_pair(s_b + s * Cfg::kBBytes, &tm_b, bar, kb * kGemmBK, n_blk * BN + rank * (BN / 2));
          if (++s == kStages) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = make_idesc_bf16_f32(256, BN, 0, 0);
      int s = 0;
      uint32_t ph = 0;
      int local = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += n_pairs, ++local) {
        const int acc = local & 1;
        const uint32_t acc_ph = (local >> 1) & 1;
        if (!mbar_wait_cluster(&acc_empty[acc], acc_ph ^ 1u, abort_flag, kKernelGemm, 12)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * Cfg::kAccStride);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_flag, kKernelGemm, 13)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t a_addr = smem_u32(s_a + s * Cfg::kABytes);
          const uint32_t b_addr = smem_u32(s_b + s * Cfg::kBBytes);
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k)
            umma_bf16_ss_pair(d_tmem, make_sdesc_sw128(a_addr + k * 32, 16, 1024),
                              make_sdesc_sw128(b_addr + k * 32, 16, 1024), idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit_pair(&empty[s], 0x3);
          if (++s == kStages) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(&acc_full[acc], 0x3);
      }
      umma_commit(drain);
      mbar_drain_wait(drain, 0);
    }
  } else {
    // Two warps per TMEM lane quadrant; each covers one half of the tile's columns.
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = static_cast<int>(rank) * 128 + quad * 32 + lane;
    float4* epi_stage = reinterpret_cast<float4*>(reinterpret_cast<uint8_t*>(full) + 256) + (warp - 2) * 256;
    const uint32_t acc_empty_leader0 = cluster_map_to_rank(&acc_empty[0], 0);
    const uint32_t acc_empty_leader1 = cluster_map_to_rank(&acc_empty[1], 0);
    int local = 0;
    for (int tile = pair; tile < num_tiles; tile += n_pairs, ++local) {
      const int m_blk = tile / p.n_blocks;
      const int n_blk = tile % p.n_blocks;
      const int acc = local & 1;
      const uint32_t acc_ph = (local >> 1) & 1;
      const int row = m_blk * 256 + row_in_tile;
      EpiPrefetch<BN, EPI> pre;
      gemm_epi_prefetch<BN, EPI>(p, row - lane, n_blk, half, pre);
      if (!mbar_wait(&acc_full[acc], acc_ph, abort_flag, kKernelGemm, 14)) break;
      tc_fence_after_sync();
      const uint32_t t_row =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * Cfg::kAccStride);
      gemm_epilogue_tile<BN, EPI>(p, row - lane, n_blk, half, t_row, epi_stage, pre);
      tc_fence_before_sync();
      mbar_arrive_cluster(acc ? acc_empty_leader1 : acc_empty_leader0);
    }
    if constexpr (is_rs_epi<EPI>() || EPI == kEpiBiasPeers) fence_acq_rel_sys();
  }

  if (*abort_flag && threadIdx.x == 0) {
    // A wait gave up: give TMA loads still in flight into this CTA's shared memory time to land.
    const uint64_t t0 = global_timer_ns();
    while (global_timer_ns() - t0 < 200000ull) {
    }
  }
  __syncthreads();
  cluster_sync_all();  // no CTA leaves while its pair may still arrive on its barriers
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
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
                                    GemmSmem<BN, EPI>::kBytes);
  });
  if (attr_err != cudaSuccess) return attr_err;
  return launch_pdl(gemm_tc_kernel<BN, EPI>, dim3(grid), dim3(kGemmThreads), GemmSmem<BN, EPI>::kBytes, stream, ta,
                    tb, p);
}

template <int BN, int EPI>
static cudaError_t launch_gemm2_t(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int grid,
                                  cudaStream_t stream) {
  using Cfg = Gemm2Cfg<BN>;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(gemm_tc2_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    gemm2_smem_bytes<BN, EPI>());
  });
  if (attr_err != cudaSuccess) return attr_err;
  return launch_pdl(gemm_tc2_kernel<BN, EPI>, dim3(grid), dim3(kGemmThreads), gemm2_smem_bytes<BN, EPI>(), stream,
                    ta, tb, p);
}

template <int BN>
static cudaError_t dispatch_epi2(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int grid,
                                 cudaStream_t stream) {
  switch (epi) {
    case kEpiBias:
      return launch_gemm2_t<BN, kEpiBias>(ta, tb, p, grid, stream);
    case kEpiBiasGelu:
      return launch_gemm2_t<BN, kEpiBiasGelu>(ta, tb, p, grid, stream);
    case kEpiResidual:
      return launch_gemm2_t<BN, kEpiResidual>(ta, tb, p, grid, stream);
    case kEpiResidualZero:
      return launch_gemm2_t<BN, kEpiResidualZero>(ta, tb, p, grid, stream);
    case kEpiStoreF32:
      return launch_gemm2_t<BN, kEpiStoreF32>(ta, tb, p, grid, stream);
    case kEpiRsResidual:
      return launch_gemm2_t<BN, kEpiRsResidual>(ta, tb, p, grid, stream);
    case kEpiRsResidualZero:
      return launch_gemm2_t<BN, kEpiRsResidualZero>(ta, tb, p, grid, stream);
    case kEpiBiasPeers:
      return launch_gemm2_t<BN, kEpiBiasPeers>(ta, tb, p, grid, stream);
    default:
      return cudaErrorInvalidValue;
  }
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
    case kEpiRsResidual:
      return launch_gemm_t<BN, kEpiRsResidual>(ta, tb, p, grid, stream);
    case kEpiRsResidualZero:
      return launch_gemm_t<BN, kEpiRsResidualZero>(ta, tb, p, grid, stream);
    case kEpiBiasPeers:
      return launch_gemm_t<BN, kEpiBiasPeers>(ta, tb, p, grid, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

constexpr int kTilePair = 0x10000;  // tile code flag: 2-SM (CTA pair) variant

// Picks the tile: the fraction of SM slots the tiles fill (waves rounded up) weighted by how well
// the tile shape keeps the tensor core fed (operand bytes per MMA work; the 2-SM pair loads 1.5x
// fewer bytes per FLOP and runs a deeper ring). The pair's advantage is in the main loop; its
// cluster launch and two-CTA handshakes are a fixed cost, so it only gets the bonus once a CTA
// pair runs at least kPairMinKBlocks k-blocks (k-blocks per tile x waves) — on the 4096-token
// C2 GEMMs (12-48 k-blocks per CTA) the one-CTA tiles measured 5-10% faster. 192-wide tiles exist
// for the D=768 projections: 768 = 4 x 192 fills a wave at M=4096 where 256-wide tiles leave a
// third of the SMs idle.
int gemm_pick_tile(int M, int N, int K, int sm_count) {
  constexpr long kPairMinKBlocks = 64;
  struct Cand {
    int code;
    int bn;
    int rows;
    int slots;
    double intensity;
  };
  const Cand cands[5] = {{kTilePair | 256, 256, 256, sm_count / 2, 1.15},
                         {kTilePair | 192, 192, 256, sm_count / 2, 1.12},
                         {256, 256, kGemmBM, sm_count, 1.0},
                         {192, 192, kGemmBM, sm_count, 0.97},
                         {128, 128, kGemmBM, sm_count, 0.85}};
  const long k_blocks = (K + kGemmBK - 1) / kGemmBK;
  int best = 128;
  double best_score = -1.0;
  for (const Cand& c : cands) {
    if (c.bn != 128 && N % c.bn != 0) continue;
    const long tiles = static_cast<long>((M + c.rows - 1) / c.rows) * ((N + c.bn - 1) / c.bn);
    const long waves = (tiles + c.slots - 1) / c.slots;
    const bool pair = (c.code & kTilePair) != 0;
    const double intensity = (pair && k_blocks * waves < kPairMinKBlocks) ? 0.95 : c.intensity;
    const double score = intensity * static_cast<double>(tiles) / static_cast<double>(waves * c.slots);
    if (score > best_score + 1e-9) {
      best = c.code;
      best_score = score;
    }
  }
  return best;
}

cudaError_t launch_gemm(const __nv_bfloat16* A, const __nv_bfloat16* W, const __nv_bfloat16* bias, int64_t M,
                        int64_t N, int64_t K, int epi, void* out, int64_t ldo, const uint8_t* row_mask, int tile,
                        cudaStream_t stream, void* const* peer_out = nullptr, int world = 1, int rank = 0,
                        int64_t rows_per_rank = 0, int64_t peer_col = 0) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = device_sm_count(dev);
  if (tile == 0) tile = gemm_pick_tile(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), sms);
  const bool pair = (tile & kTilePair) != 0;
  const int bn = tile & 0xFFFF;
  CUtensorMap ta, tb;
  cudaError_t e = make_tmap_bf16_2d(&ta, A, K, M, K * 2, kGemmBK, kGemmBM);
  if (e != cudaSuccess) return e;
  e = make_tmap_bf16_2d(&tb, W, K, N, K * 2, kGemmBK, pair ? bn / 2 : bn);
  if (e != cudaSuccess) return e;
  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  for (int r = 0; peer_out != nullptr && r < world; ++r) p.peer_out[r] = peer_out[r];
  p.world = world;
  p.rank = rank;
  p.rows_per_rank = static_cast<int>(rows_per_rank);
  p.peer_col = static_cast<int>(peer_col);
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
  if (pair) {
    const long tiles = static_cast<long>((M + 255) / 256) * p.n_blocks;
    const long pairs = tiles < sms / 2 ? tiles : sms / 2;
    const int grid = static_cast<int>(2 * pairs);
    if (bn == 256) return dispatch_epi2<256>(epi, ta, tb, p, grid, stream);
    if (bn == 192) return dispatch_epi2<192>(epi, ta, tb, p, grid, stream);
    return cudaErrorInvalidValue;
  }
  const long tiles = static_cast<long>(p.m_blocks) * p.n_blocks;
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);
  if (bn == 256) return dispatch_epi<256>(epi, ta, tb, p, grid, stream);
  if (bn == 192) return dispatch_epi<192>(epi, ta, tb, p, grid, stream);
  return dispatch_epi<128>(epi, ta, tb, p, grid, stream);
}

// ---------------------------------------------------------------------------------------------
// GEMM + residual + LayerNorm (kEpiResidualLn / kEpiResidualZeroLn): clusters of N / BN CTAs.
// ---------------------------------------------------------------------------------------------
// Picks the column tile of the LayerNorm-fused GEMM. The cluster spans the row (cs = N / bn <= 8
// CTAs) and each row's statistics are summed in an order fixed by bn, so the choice depends on N
// alone — never on M — to keep every row's output independent of how many rows share the launch
// (batch shards give the same bits as the full batch): n <= 256 takes one CTA; otherwise a
// power-of-two cluster is preferred, then the widest tile. *recommended is 0 for every width: on
// B200 the fused launch measured slower than the GEMM followed by the separate LayerNorm kernel
// (C2 1.668 vs 1.637 ms per forward, C3 4.70 vs 4.46, C1 0.228 vs 0.198). Its epilogue runs its
// passes back to back on one 128-row tile per CTA (load and update the residual, merge and exchange
// the row statistics, store residual and LayerNorm rows: 4.7 + 3.3 + 2.4 us at C2's out_proj), while
// the separate LayerNorm, launched with programmatic dependent launch, overlaps the GEMM's tail and
// adds about 3 us; with 256-wide tiles the exchange and staging buffers also leave a 3-deep ring.
bool gemm_ln_plan(int64_t M, int64_t N, int64_t K, int sms, int* bn_out, int* cs_out, int* recommended) {
  (void)sms;
  if (M <= 0 || N <= 0 || K <= 0 || N % 32 != 0) return false;
  int bn = 0, cs = 0;
  if (N <= 256) {
    bn = N <= 128 ? 128 : (N <= 192 ? 192 : 256);
    cs = 1;
  } else {
    const int cand[3] = {256, 192, 128};
    for (int pow2 = 1; pow2 >= 0 && cs == 0; --pow2) {
      for (int i = 0; i < 3 && cs == 0; ++i) {
        if (N % cand[i] != 0) continue;
        const int c = static_cast<int>(N / cand[i]);
        if (c > kLnMaxCluster || (pow2 && (c & (c - 1)) != 0)) continue;
        bn = cand[i];
        cs = c;
      }
    }
    if (cs == 0) return false;
  }
  if (bn_out) *bn_out = bn;
  if (cs_out) *cs_out = cs;
  if (recommended) *recommended = 0;
  return true;
}

template <int BN, int EPI>
static cudaError_t launch_gemm_ln_t(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int cs,
                                    cudaStream_t stream) {
  static std::once_flag once[64];
  static std::atomic<int> max_clusters[64][kLnMaxCluster + 1];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    GemmSmem<BN, EPI>::kBytes);
  });
  if (attr_err != cudaSuccess) return attr_err;
  cudaLaunchConfig_t config = {};
  config.blockDim = dim3(kGemmThreads);
  config.dynamicSmemBytes = GemmSmem<BN, EPI>::kBytes;
  config.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cs);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attr;
  config.numAttrs = 2;
  // The kernel is persistent: at most as many clusters as can be resident at once.
  std::atomic<int>& cached = max_clusters[dev & 63][cs];
  int resident = cached.load();
  if (resident == 0) {
    config.gridDim = dim3(static_cast<unsigned>(cs * p.m_blocks));
    const cudaError_t e = cudaOccupancyMaxActiveClusters(&resident, gemm_tc_kernel<BN, EPI>, &config);
    if (e != cudaSuccess) return e;
    if (resident <= 0) return cudaErrorInvalidConfiguration;
    cached.store(resident);
  }
  const int clusters = p.m_blocks < resident ? p.m_blocks : resident;
  config.gridDim = dim3(static_cast<unsigned>(cs * clusters));
  return cudaLaunchKernelEx(&config, gemm_tc_kernel<BN, EPI>, ta, tb, p);
}

template <int BN>
static cudaError_t dispatch_ln(bool zero_masked, const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p,
                               int cs, cudaStream_t stream) {
  return zero_masked ? launch_gemm_ln_t<BN, kEpiResidualZeroLn>(ta, tb, p, cs, stream)
                     : launch_gemm_ln_t<BN, kEpiResidualLn>(ta, tb, p, cs, stream);
}

// resid[M, N] (fp32) += A W^T + bias on kept rows (kept rows only, or kept rows and zeros when
// zero_masked), then ln_out[M, N] = LayerNorm(resid) with gamma / beta / eps, in one launch.
cudaError_t launch_gemm_ln(const __nv_bfloat16* A, const __nv_bfloat16* W, const __nv_bfloat16* bias, int64_t M,
                           int64_t N, int64_t K, bool zero_masked, float* resid, const uint8_t* row_mask,
                           const __nv_bfloat16* gamma, const __nv_bfloat16* beta, float eps, __nv_bfloat16* ln_out,
                           cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = device_sm_count(dev);
  int bn = 0, cs = 0;
  if (!gemm_ln_plan(M, N, K, sms, &bn, &cs, nullptr)) return cudaErrorInvalidValue;
  CUtensorMap ta, tb;
  cudaError_t e = make_tmap_bf16_2d(&ta, A, K, M, K * 2, kGemmBK, kGemmBM);
  if (e != cudaSuccess) return e;
  e = make_tmap_bf16_2d(&tb, W, K, N, K * 2, kGemmBK, bn);
  if (e != cudaSuccess) return e;
  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.out = resid;
  p.ldo = N;
  p.bias = bias;
  p.row_mask = row_mask;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.m_blocks = static_cast<int>((M + kGemmBM - 1) / kGemmBM);
  p.n_blocks = static_cast<int>((N + bn - 1) / bn);
  p.k_blocks = static_cast<int>((K + kGemmBK - 1) / kGemmBK);
  p.world = 1;
  p.ln_gamma = gamma;
  p.ln_beta = beta;
  p.ln_out = ln_out;
  p.ln_eps = eps;
  if (p.n_blocks != cs) return cudaErrorInvalidValue;
  if (bn == 256) return dispatch_ln<256>(zero_masked, ta, tb, p, cs, stream);
  if (bn == 192) return dispatch_ln<192>(zero_masked, ta, tb, p, cs, stream);
  return dispatch_ln<128>(zero_masked, ta, tb, p, cs, stream);
}

}  // namespace b2
