// Flash-style multi-head self-attention forward on tcgen05 tensor cores.
//
// Computes, per batch b, head h and query q (BaselineSelfAttention.forward,
// transformer_benchmark/models.py:55-75):
//   s_k  = (q . k_k) * head_dim^-0.5
//   s_k  = -inf  where causal and k > q (:57-61), or where key k is padding (:63-66)
//   p    = softmax(s) in fp32 (:69)
//   ctx  = p . V, written as bf16 straight into the token-major [B*S, H*hd] context (:70-75)
// without materialising the [B, H, S, S] score tensor: scores stream through TMEM tile by tile
// with an online (running-max) softmax. Padding follows generate_random_case's prefix masks
// (transformer_benchmark/cases.py:87-97): key k of batch b is valid iff k < kv_len[b]. Query
// tiles that lie wholly past kv_len[b] are skipped; their context rows are never read because
// the out_proj epilogue keeps the residual for masked rows (models.py:78-79).
//
// Q, K and V are read in place from the packed QKV projection output [B*S, ld] (head h of Q at
// columns q_col + h*hd, likewise K and V), by TMA with 128-byte swizzle, 64 columns per box.
//
// CTA = one (b, h, 128-query tile); 10 warps:
//   warp 0      TMA producer: Q once, then K_j and V_j (128 keys each) into 2-stage rings.
//   warp 1      TMEM allocator and UMMA issuer: S_j = Q K_j^T (M=128, N=128, K=hd) into one of
//               two TMEM score buffers, then O_j = P_j V_j (M=128, N=hd, K=128) into one of two
//               TMEM output buffers; S_{j+1} is issued before O_j so the tensor core works while
//               the softmax warps are busy.
//   warps 2..9  softmax: TMEM lane quadrant (warp % 4) gives the query row, warp group (0/1)
//               gives which 64 of the 128 key columns (and which half of hd) the thread owns.
//               Row maxima are exchanged between the two groups through shared memory; the
//               unnormalised probabilities are written as bf16 in the K-major SW128 layout the
//               P V MMA reads; O accumulates in registers with the running-max correction.
// Query tiles are issued heaviest-first (causal rows near the end of the sequence see the most
// keys), which keeps the tail of the grid short.
#include <mutex>

#pragma once
#include "b2_common.cuh"

namespace b2 {

struct AttnParams {
  __nv_bfloat16* ctx;
  int64_t ld_ctx;
  const int32_t* kv_len;
  int B, S, H;
  int q_col, k_col, v_col;
  int causal;
  float scale_log2;  // head_dim^-0.5 * log2(e)
  int n_q_tiles;
};

constexpr int kAttnThreads = 320;
constexpr int kAttnSoftmaxThreads = 256;

template <int HD>
struct AttnCfg {
  static constexpr int kBoxBytes = 128 * 128;  // one 128-row x 64-column bf16 box
  static constexpr int kBoxes = HD / 64;
  static constexpr int kTileBytes = 128 * HD * 2;
  static constexpr int kKvStages = 2;
  static constexpr int kPBufs = HD == 128 ? 1 : 2;
  static constexpr int kPBytes = 128 * 128 * 2;
  // head_dim 64: the P.V MMA also produces the softmax row sums. Each V stage is followed by a
  // 64-column block of bf16 ones (the MN-major operand's next N block, LBO = one box), the MMA
  // runs with N = 64 + 16, and columns 64..79 of O_j hold sum_k P_j[r, k] in fp32 (the sum of
  // exactly the bf16 weights that multiply V). head_dim 128 has no shared-memory room for that
  // and sums in registers.
  static constexpr bool kTcRowSum = HD == 64;
  static constexpr int kVStageBytes = kTileBytes + (kTcRowSum ? kBoxBytes : 0);
  static constexpr int kON = HD + (kTcRowSum ? 16 : 0);
  static constexpr int kTmemCols = 512;
  static constexpr int kSCol = 0;
  static constexpr int kOCol = 256;
  static constexpr int kOStride = 128;
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kTileBytes;
  static constexpr int kOffV = kOffK + kKvStages * kTileBytes;
  static constexpr int kOffP = kOffV + kKvStages * kVStageBytes;
  static constexpr int kOffRed = kOffP + kPBufs * kPBytes;             // float [2][2][128] row maxima
  static constexpr int kOffSum = kOffRed + 2 * 2 * 128 * 4;            // float [2][128] row sums
  static constexpr int kOffBar = kOffSum + 2 * 128 * 4;
  static constexpr int kBarrierBytes = 256;
  static constexpr int kSmemBytes = kOffBar + kBarrierBytes + 1024;
};

// Softmax-warp wait: once any wait of this thread gave up (`alive` false) later waits are
// skipped, so the warp still runs its remaining iterations and every named barrier stays matched.
__device__ __forceinline__ void softmax_wait(uint64_t* bar, uint32_t parity, uint32_t site, bool& alive,
                                             volatile int* abort_flag) {
  if (alive && !mbar_wait(bar, parity, abort_flag, kKernelAttention, site)) alive = false;
}

// O_acc = O_acc * a + O_i, where O_i = P_i V_i sits in TMEM output buffer (i & 1); `t_lane` is
// this thread's TMEM lane at column 0, `grp` its hd half. With tensor-core row sums the running
// sum l_acc gets the same update from the row-sum column of O_i.
template <int HD>
__device__ __forceinline__ void accumulate_o(float (&o_acc)[HD / 2], float& l_acc, int i, float a,
                                             uint64_t* o_full, uint64_t* o_empty, uint32_t t_lane, int grp,
                                             int lane, bool& alive, volatile int* abort_flag) {
  using Cfg = AttnCfg<HD>;
  const int ob = i & 1;
  softmax_wait(&o_full[ob], (i >> 1) & 1, 9, alive, abort_flag);
  tc_fence_after_sync();
  const uint32_t t_buf = t_lane + Cfg::kOCol + ob * Cfg::kOStride;
  const uint32_t t = t_buf + grp * (HD / 2);
  if constexpr (Cfg::kTcRowSum) l_acc = fmaf(l_acc, a, tmem_load_1col(t_buf + HD));
#pragma unroll
  for (int cc = 0; cc < HD / 64; ++cc) {
    float v[32];
    tmem_load_32cols(t + cc * 32, v);
#pragma unroll
    for (int k = 0; k < 32; ++k) o_acc[cc * 32 + k] = fmaf(o_acc[cc * 32 + k], a, v[k]);
  }
  tc_fence_before_sync();
  __syncwarp();
  if (lane == 0) mbar_arrive(&o_empty[ob]);
}

template <int HD>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, const AttnParams p) {
  using Cfg = AttnCfg<HD>;
  constexpr int kBoxBytes = Cfg::kBoxBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_q = smem + Cfg::kOffQ;
  uint8_t* s_k = smem + Cfg::kOffK;
  uint8_t* s_v = smem + Cfg::kOffV;
  uint8_t* s_p = smem + Cfg::kOffP;
  float* red_max = reinterpret_cast<float*>(smem + Cfg::kOffRed);
  float* red_sum = reinterpret_cast<float*>(smem + Cfg::kOffSum);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* s_empty = bars + 11; // [2]
  uint64_t* p_full = bars + 13;  // [2]
  uint64_t* p_empty = bars + 15; // [2]
  uint64_t* o_full = bars + 17;  // [2]
  uint64_t* o_empty = bars + 19; // [2]
  uint64_t* drain = bars + 21;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 22);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int b = bh / p.H;
  const int h = bh % p.H;
  const int qt = p.n_q_tiles - 1 - static_cast<int>(blockIdx.y);
  const int q0 = qt * 128;
  const int kv_len = p.kv_len != nullptr ? p.kv_len[b] : p.S;
  if (q0 >= kv_len || kv_len <= 0) return;  // uniform for the CTA: nothing allocated yet
  const int kv_tiles_len = (kv_len + 127) / 128;
  const int n_kv = p.causal ? min(qt + 1, kv_tiles_len) : kv_tiles_len;
  const int row_base = b * p.S;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 8);
      mbar_init(&p_full[i], 8);
      mbar_init(&p_empty[i], 1);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 8);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tm_qkv);
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  if constexpr (Cfg::kTcRowSum) {
    // bf16 1.0 everywhere in the ones blocks (so the swizzle does not matter), made visible to
    // the tensor core's async-proxy reads.
    for (int st = 0; st < Cfg::kKvStages; ++st) {
      uint4* ones = reinterpret_cast<uint4*>(s_v + st * Cfg::kVStageBytes + Cfg::kTileBytes);
      for (int i = threadIdx.x; i < kBoxBytes / 16; i += kAttnThreads)
        ones[i] = make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u);
    }
    fence_proxy_async_smem();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait_previous_grid();
  pdl_allow_next_grid();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const int qc = p.q_col + h * HD;
      const int kc = p.k_col + h * HD;
      const int vc = p.v_col + h * HD;
      mbar_arrive_expect_tx(q_full, Cfg::kTileBytes);
#pragma unroll
      for (int c = 0; c < Cfg::kBoxes; ++c) tma_load_2d(s_q + c * kBoxBytes, &tm_qkv, q_full, qc + c * 64, row_base + q0);
      int issued_k = 0, issued_v = 0;
      bool ok = true;
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        const int krow = row_base + j * 128;
        if (!mbar_wait(&k_empty[st], ph ^ 1u, abort_flag, kKernelAttention, 1)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&k_full[st], Cfg::kTileBytes);
#pragma unroll
        for (int c = 0; c < Cfg::kBoxes; ++c)
          tma_load_2d(s_k + st * Cfg::kTileBytes + c * kBoxBytes, &tm_qkv, &k_full[st], kc + c * 64, krow);
        ++issued_k;
        if (!mbar_wait(&v_empty[st], ph ^ 1u, abort_flag, kKernelAttention, 2)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&v_full[st], Cfg::kTileBytes);
#pragma unroll
        for (int c = 0; c < Cfg::kBoxes; ++c)
          tma_load_2d(s_v + st * Cfg::kVStageBytes + c * kBoxBytes, &tm_qkv, &v_full[st], vc + c * 64, krow);
        ++issued_v;
      }
      if (!ok) {
        // Let copies in flight land: Q, and the last (up to two) K and V tiles.
        const uint64_t t0 = global_timer_ns();
        auto drain_wait = [&](uint64_t* bar, uint32_t par) {
          while (!mbar_try_wait(bar, par) && global_timer_ns() - t0 < kWaitTimeoutNs) {
          }
        };
        drain_wait(q_full, 0);
        for (int j = issued_k - 1; j >= 0 && j >= issued_k - 2; --j) drain_wait(&k_full[j & 1], (j >> 1) & 1);
        for (int j = issued_v - 1; j >= 0 && j >= issued_v - 2; --j) drain_wait(&v_full[j & 1], (j >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------- UMMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16_f32(128, 128, 0, 0);
      constexpr uint32_t idesc_o = make_idesc_bf16_f32(128, Cfg::kON, 0, 1);
      bool ok = mbar_wait(q_full, 0, abort_flag, kKernelAttention, 3);
      if (ok) tc_fence_after_sync();
      const uint32_t q_addr = smem_u32(s_q);
      for (int j = 0; j <= n_kv && ok; ++j) {
        if (j < n_kv) {
          const int st = j & 1;
          const uint32_t ph = (j >> 1) & 1;
          if (!mbar_wait(&k_full[st], ph, abort_flag, kKernelAttention, 4)) break;
          if (!mbar_wait(&s_empty[st], ph ^ 1u, abort_flag, kKernelAttention, 5)) break;
          tc_fence_after_sync();
          const uint32_t d = tmem_base + Cfg::kSCol + st * 128;
          const uint32_t k_addr = smem_u32(s_k + st * Cfg::kTileBytes);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kBoxBytes + (kk & 3) * 32;
            umma_bf16_ss(d, make_sdesc_sw128(q_addr + off, 16, 1024), make_sdesc_sw128(k_addr + off, 16, 1024),
                         idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[st]);
          umma_commit(&k_empty[st]);
        }
        if (j >= 1) {
          const int i = j - 1;
          const int st = i & 1;
          const uint32_t ph = (i >> 1) & 1;
          const int pb = i % Cfg::kPBufs;
          const uint32_t pph = (i / Cfg::kPBufs) & 1;
          if (!mbar_wait(&v_full[st], ph, abort_flag, kKernelAttention, 6)) break;
          if (!mbar_wait(&p_full[pb], pph, abort_flag, kKernelAttention, 7)) break;
          if (!mbar_wait(&o_empty[st], ph ^ 1u, abort_flag, kKernelAttention, 8)) break;
          tc_fence_after_sync();
          const uint32_t d = tmem_base + Cfg::kOCol + st * Cfg::kOStride;
          const uint32_t p_addr = smem_u32(s_p + pb * Cfg::kPBytes);
          const uint32_t v_addr = smem_u32(s_v + st * Cfg::kVStageBytes);
#pragma unroll
          for (int kk = 0; kk < 128 / 16; ++kk) {
            const uint64_t a_desc = make_sdesc_sw128(p_addr + (kk >> 2) * kBoxBytes + (kk & 3) * 32, 16, 1024);
            const uint64_t b_desc = make_sdesc_sw128(v_addr + kk * 2048, kBoxBytes, 1024);
            umma_bf16_ss(d, a_desc, b_desc, idesc_o, kk > 0 ? 1u : 0u);
          }
          umma_commit(&o_full[st]);
          umma_commit(&v_empty[st]);
          umma_commit(&p_empty[pb]);
        }
      }
      umma_commit(drain);
      const uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(drain, 0) && global_timer_ns() - t0 < kWaitTimeoutNs) {
      }
    }
  } else {
    // ---------------- softmax / output warps ----------------
    const int sw = warp - 2;           // 0..7
    const int grp = sw >> 2;           // key-column half / hd half
    const int quad = warp & 3;         // TMEM lane quadrant
    const int r = quad * 32 + lane;    // row in the query tile
    const int query = q0 + r;
    constexpr int kOHalf = HD / 2;
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    const float c = p.scale_log2;

    float o_acc[kOHalf];
#pragma unroll
    for (int k = 0; k < kOHalf; ++k) o_acc[k] = 0.f;
    float m_run = -INFINITY;  // running row maximum of raw scores
    float l_run = 0.f;        // register row sum (head_dim 128): this thread's 64 columns
    float l_acc = 0.f;        // tensor-core row sum (head_dim 64): whole row
    float alpha_prev = 0.f;
    bool alive = true;  // false after any wait gave up; the loop still runs to keep barriers matched

#pragma unroll 1
    for (int j = 0; j < n_kv; ++j) {
      const int sb = j & 1;
      softmax_wait(&s_full[sb], (j >> 1) & 1, 10, alive, abort_flag);
      tc_fence_after_sync();
      float s[64];
      tmem_load_32cols(t_lane + Cfg::kSCol + sb * 128 + grp * 64, s);
      tmem_load_32cols(t_lane + Cfg::kSCol + sb * 128 + grp * 64 + 32, s + 32);
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[sb]);

      if (j == n_kv - 1) {
        // Keys [key0, key0 + n_valid) of this thread's 64 are visible to its query row.
        const int key0 = j * 128 + grp * 64;
        const int limit = p.causal ? min(kv_len, query + 1) : kv_len;
        const int n_valid = limit - key0;
#pragma unroll
        for (int k = 0; k < 64; ++k) s[k] = (k < n_valid) ? s[k] : -INFINITY;
      }
      float pmax = max3f(s[0], s[1], s[2]);
#pragma unroll
      for (int k = 3; k < 63; k += 2) pmax = max3f(pmax, s[k], s[k + 1]);
      pmax = fmaxf(pmax, s[63]);
      float* red = red_max + (j & 1) * 256;
      red[grp * 128 + r] = pmax;
      named_barrier_sync(1, kAttnSoftmaxThreads);
      const float omax = red[(grp ^ 1) * 128 + r];
      const float m_new = fmaxf(m_run, fmaxf(pmax, omax));
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = fast_exp2((m_run - m_use) * c);
      const float neg_mc = -m_use * c;

      // P_j -> shared memory, K-major SW128: atom `grp` holds keys [64*grp, 64*grp+64) of all
      // 128 rows; row r at (r/8)*1024 + (r%8)*128, 16-byte chunk ch stored at chunk ch ^ (r%8).
      // Each 8-key chunk is stored as soon as it is computed, which keeps register use low.
      const int pb = j % Cfg::kPBufs;
      softmax_wait(&p_empty[pb], ((j / Cfg::kPBufs) & 1) ^ 1u, 11, alive, abort_flag);
      uint8_t* prow = s_p + pb * Cfg::kPBytes + grp * kBoxBytes + (r >> 3) * 1024 + (r & 7) * 128;
      float lsum = 0.f;
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float e0 = fast_exp2(fmaf(s[8 * ch + 2 * k], c, neg_mc));
          const float e1 = fast_exp2(fmaf(s[8 * ch + 2 * k + 1], c, neg_mc));
          if constexpr (!Cfg::kTcRowSum) lsum += e0 + e1;
          w[k] = pack_bf16x2(e0, e1);
        }
        *reinterpret_cast<uint4*>(prow + ((ch ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      l_run = fmaf(l_run, alpha, lsum);
      m_run = m_new;
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[pb]);

      if (j >= 1)
        accumulate_o<HD>(o_acc, l_acc, j - 1, alpha_prev, o_full, o_empty, t_lane, grp, lane, alive, abort_flag);
      alpha_prev = alpha;
    }
    if (n_kv >= 1)
      accumulate_o<HD>(o_acc, l_acc, n_kv - 1, alpha_prev, o_full, o_empty, t_lane, grp, lane, alive, abort_flag);

    float l_tot = l_acc;
    if constexpr (!Cfg::kTcRowSum) {
      red_sum[grp * 128 + r] = l_run;
      named_barrier_sync(1, kAttnSoftmaxThreads);
      l_tot = l_run + red_sum[(grp ^ 1) * 128 + r];
    }
    const float inv = l_tot > 0.f ? 1.0f / l_tot : 0.f;
    if (query < p.S) {
      uint4* dst = reinterpret_cast<uint4*>(p.ctx + static_cast<int64_t>(row_base + query) * p.ld_ctx + h * HD +
                                            grp * kOHalf);
#pragma unroll
      for (int v = 0; v < kOHalf / 8; ++v) {
        dst[v] = make_uint4(pack_bf16x2(o_acc[8 * v] * inv, o_acc[8 * v + 1] * inv),
                            pack_bf16x2(o_acc[8 * v + 2] * inv, o_acc[8 * v + 3] * inv),
                            pack_bf16x2(o_acc[8 * v + 4] * inv, o_acc[8 * v + 5] * inv),
                            pack_bf16x2(o_acc[8 * v + 6] * inv, o_acc[8 * v + 7] * inv));
      }
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

template <int HD>
static cudaError_t launch_attention_t(const CUtensorMap& tm, const AttnParams& p, cudaStream_t stream) {
  using Cfg = AttnCfg<HD>;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(attention_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    Cfg::kSmemBytes);
  });
  if (attr_err != cudaSuccess) return attr_err;
  dim3 grid(p.B * p.H, p.n_q_tiles);
  return launch_pdl(attention_tc_kernel<HD>, grid, dim3(kAttnThreads), Cfg::kSmemBytes, stream, tm, p);
}

static cudaError_t launch_attention_pair(const CUtensorMap& tm, const AttnParams& p, cudaStream_t stream);

cudaError_t launch_attention(const __nv_bfloat16* qkv, int64_t ld_qkv, int64_t q_col, int64_t k_col, int64_t v_col,
                             int64_t B, int64_t S, int64_t H, int64_t hd, const int32_t* kv_len, int causal,
                             float scale, __nv_bfloat16* ctx, int64_t ld_ctx, cudaStream_t stream) {
  CUtensorMap tm;
  cudaError_t e = make_tmap_bf16_2d(&tm, qkv, static_cast<uint64_t>(ld_qkv), static_cast<uint64_t>(B * S),
                                    static_cast<uint64_t>(ld_qkv) * 2, 64, 128);
  if (e != cudaSuccess) return e;
  AttnParams p;
  p.ctx = ctx;
  p.ld_ctx = ld_ctx;
  p.kv_len = kv_len;
  p.B = static_cast<int>(B);
  p.S = static_cast<int>(S);
  p.H = static_cast<int>(H);
  p.q_col = static_cast<int>(q_col);
  p.k_col = static_cast<int>(k_col);
  p.v_col = static_cast<int>(v_col);
  p.causal = causal;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.n_q_tiles = static_cast<int>((S + 127) / 128);
  if (hd == 64) return launch_attention_pair(tm, p, stream);
  if (hd == 128) return launch_attention_t<128>(tm, p, stream);
  return cudaErrorInvalidValue;
}

}  // namespace b2
