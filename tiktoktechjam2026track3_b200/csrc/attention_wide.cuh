// Flash attention forward, head_dim 128, one query tile per CTA with three score buffers (the
// paths of BaselineSelfAttention.forward, transformer_benchmark/models.py:55-75; masks as in
// attention.cuh).
//
// At head_dim 128 a 128 x 128 score tile costs as many tensor-core cycles for S = Q K^T as for
// O += P V (2 x 4.2 MFLOP) and about 1000 cycles of exponentials. A kernel with two query tiles
// per CTA and one score buffer per tile (P written over it) made S(j+1) of a tile wait for
// O += P(j) V, and its tensor pipe was idle more than half the time (41.5 % active at B=1
// S=8192). Here one query tile owns three score buffers in tensor memory (3 x 128 columns, P(j)
// written over S(j)'s first 64 once the scores are in registers) and O (128 columns): S(j+2) is
// computed while the softmax works on S(j), and the softmax never waits for a score tile.
// Measured against the two-tile kernel on one B200 (CUDA events, L2 flushed; bit-identical
// outputs before the FMA-pipe share below): B=1 S=32768 16 heads causal (C4) 4425 -> 4109 us,
// B=1 S=8192 317 -> 302 us, B=1 S=4096 2 heads 82 -> 47 us, B=1 S=1024 2 heads 26.7 -> 18.5 us;
// non-causal B=2 S=2048 unchanged (101 us). One pair in four of the exponentials on the FMA pipe
// (exp2_poly_x2) then gave 4106 -> 4077 us at C4's shape and 300 -> 293 us at S=8192 (one in two
// was slower); splitting each row's 128 keys between two softmax warps (320 threads, a row-maximum
// exchange per tile) was measured slower (4115 us). Issuing S = Q K^T and O += P V from two
// threads instead of one (a thread's back-to-back tcgen05.mma take at least ~114 clocks each at
// N <= 128, so one issuer left the tensor core idle between instructions) then gave 4005 -> 3861 us
// at C4's shape and 299 -> 282 us at S=8192, bit-identical.
//
//   warp 0      TMA: Q once (two 64-column boxes); K_j and V_j (128 keys x 128 dims, two boxes
//               each) into two 3-stage rings.
//   warp 1      TMEM allocator and issuer of S: S(0), S(1), then S(j+2) into the buffer P(j-1)
//               occupied once P(j) is published (which means O += P(j-1) V completed: the softmax
//               waits for it before storing P(j)).
//   warp 6      issuer of O += P(j) V_j once P(j) is published.
//   warps 2..5  softmax, one query row per thread (warp % 4 = TMEM lane quadrant): row maximum,
//               exp2(c s - c m) into registers as bf16 pairs, then (after O += P(j-1) V has landed)
//               the pairs into P and, when the reference maximum moved by more than 2^8, O rescaled.
// Tensor memory (512 columns): S_b at 128 b (b = j mod 3) with P_b over its first 64 columns, O at
// 384. One CTA per SM (224 KB of shared memory).
#pragma once
#include "b2_common.cuh"
#include "attention.cuh"

namespace b2 {

struct AttnWideCfg {
  static constexpr int kThreads = 224;
  static constexpr int kPvWarp = 6;  // O += P V issuer (warps 2..5 are the softmax)
  static constexpr int kBoxBytes = 128 * 128;     // 128 rows x 64 bf16 columns (one TMA box)
  static constexpr int kTileBytes = 2 * kBoxBytes;  // 128 rows x 128 bf16 columns
  static constexpr int kStages = 3;
  static constexpr int kBufs = 3;                 // score buffers in tensor memory
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kTileBytes;
  static constexpr int kOffV = kOffK + kStages * kTileBytes;
  static constexpr int kOffBar = kOffV + kStages * kTileBytes;
  static constexpr int kSmemBytes = kOffBar + 256 + 1024;
  static constexpr int kTmemCols = 512;
  static constexpr int kOCol = kBufs * 128;
  // bit k: pair k of every 4 takes 2^x on the FMA pipe (exp2_poly_x2) instead of the exponential unit
  static constexpr int kPolyPairs = 0x1;
  static_assert(kSmemBytes <= 232448, "shared memory per CTA");
};

__global__ void __launch_bounds__(AttnWideCfg::kThreads, 1)
    attention_wide_kernel(const __grid_constant__ CUtensorMap tm_qkv, const AttnParams p) {
  using Cfg = AttnWideCfg;
  constexpr int HD = 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_q = smem + Cfg::kOffQ;
  uint8_t* s_k = smem + Cfg::kOffK;
  uint8_t* s_v = smem + Cfg::kOffV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = q_full + 1;               // [kStages]
  uint64_t* k_empty = k_full + Cfg::kStages;   // [kStages]
  uint64_t* v_full = k_empty + Cfg::kStages;   // [kStages]
  uint64_t* v_empty = v_full + Cfg::kStages;   // [kStages]
  uint64_t* s_full = v_empty + Cfg::kStages;   // [kBufs]
  uint64_t* p_full = s_full + Cfg::kBufs;      // [kBufs]
  uint64_t* o_full = p_full + Cfg::kBufs;
  uint64_t* drain = o_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int bh, cta_row;
  attn_cta_coords(p, bh, cta_row);
  const int b = bh / p.H;
  const int h = bh % p.H;
  int y_local;
  const int rg = attn_range_of(p, cta_row, p.n_q_tiles, y_local);
  const int tile = p.n_q_tiles[rg] - 1 - y_local;  // heaviest causal tiles first
  const int qt = p.q_tile0[rg] + tile;               // absolute query tile
  const int q_end = p.q_end[rg];
  const int kv_len = p.kv_len != nullptr ? p.kv_len[b] : p.S;
  const int kv_tiles = (kv_len + 127) >> 7;
  const int n = qt * 128 < kv_len ? (p.causal ? min(qt + 1, kv_tiles) : kv_tiles) : 0;
  if (n == 0) return;  // uniform for the CTA: nothing allocated yet
  const int row_base = b * p.S;
  const int q_row0 = row_base + qt * 128;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < Cfg::kStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < Cfg::kBufs; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
    }
    mbar_init(o_full, 1);
    mbar_init(drain, 2);  // one commit from each issuer
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tm_qkv);
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
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
      mbar_arrive_expect_tx(q_full, static_cast<uint32_t>(Cfg::kTileBytes));
      tma_load_2d(s_q, &tm_qkv, q_full, qc, q_row0);
      tma_load_2d(s_q + Cfg::kBoxBytes, &tm_qkv, q_full, qc + 64, q_row0);
      int k_next = 0, v_next = 0;
      bool ok = true;
      PollTimeout poll;
      poll.reset();
      while (k_next < n || v_next < n) {
        bool progress = false;
        if (k_next < n && mbar_test_wait(&k_empty[k_next % Cfg::kStages], ((k_next / Cfg::kStages) & 1) ^ 1u)) {
          const int st = k_next % Cfg::kStages;
          uint8_t* dst = s_k + st * Cfg::kTileBytes;
          mbar_arrive_expect_tx(&k_full[st], Cfg::kTileBytes);
          tma_load_2d(dst, &tm_qkv, &k_full[st], kc, row_base + k_next * 128);
          tma_load_2d(dst + Cfg::kBoxBytes, &tm_qkv, &k_full[st], kc + 64, row_base + k_next * 128);
          ++k_next;
          progress = true;
        }
        if (v_next < n && mbar_test_wait(&v_empty[v_next % Cfg::kStages], ((v_next / Cfg::kStages) & 1) ^ 1u)) {
          const int st = v_next % Cfg::kStages;
          uint8_t* dst = s_v + st * Cfg::kTileBytes;
          mbar_arrive_expect_tx(&v_full[st], Cfg::kTileBytes);
          tma_load_2d(dst, &tm_qkv, &v_full[st], vc, row_base + v_next * 128);
          tma_load_2d(dst + Cfg::kBoxBytes, &tm_qkv, &v_full[st], vc + 64, row_base + v_next * 128);
          ++v_next;
          progress = true;
        }
        if (progress) {
          poll.reset();
        } else if (*abort_flag) {
          ok = false;
          break;
        } else if (poll.expired()) {
          record_status(kKernelAttention, 71, kReasonTimeout);
          *abort_flag = 1;
          ok = false;
          break;
        }
      }
      if (!ok) {
        // Let copies in flight land: Q and the last (up to kStages) K and V tiles.
        const uint64_t t0 = global_timer_ns();
        const uint64_t lim = wait_limit_ns();
        auto drain_wait = [&](uint64_t* bar, uint32_t par) {
          while (!mbar_try_wait(bar, par) && global_timer_ns() - t0 < lim) {
          }
        };
        drain_wait(q_full, 0);
        for (int j = k_next - 1; j >= 0 && j >= k_next - Cfg::kStages; --j)
          drain_wait(&k_full[j % Cfg::kStages], (j / Cfg::kStages) & 1);
        for (int j = v_next - 1; j >= 0 && j >= v_next - Cfg::kStages; --j)
          drain_wait(&v_full[j % Cfg::kStages], (j / Cfg::kStages) & 1);
      }
    }
  } else if (warp == 1 || warp == Cfg::kPvWarp) {
    // ---------------- UMMA issuers ----------------
    // Two threads issue: warp 1 the products S = Q K^T, warp kPvWarp the products O += P V. One
    // thread's back-to-back tcgen05.mma take at least ~114 clocks each at N <= 128 (measured on
    // B200), so with one issuer the tensor core idles between the instructions of each product;
    // two issuers keep both products in flight. Each commit tracks its own thread's MMAs only.
    if (lane == 0) {
      bool ok = true;
      if (warp == 1) {
        constexpr uint32_t idesc_s = make_idesc_bf16_f32(128, 128, 0, 0);
        const uint32_t q_addr = smem_u32(s_q);
        // S(j) into buffer j mod 3 once K_j is loaded.
        auto issue_s = [&](int j) -> bool {
          const int st = j % Cfg::kStages;
          if (!mbar_wait(&k_full[st], (j / Cfg::kStages) & 1, abort_flag, kKernelAttention, 72)) return false;
          tc_fence_after_sync();
          const uint32_t k_addr = smem_u32(s_k + st * Cfg::kTileBytes);
          const uint32_t d_s = tmem_base + (j % Cfg::kBufs) * 128;
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * Cfg::kBoxBytes + (kk & 3) * 32;
            umma_bf16_ss(d_s, make_sdesc_sw128(q_addr + off, 16, 1024), make_sdesc_sw128(k_addr + off, 16, 1024),
                         idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[j % Cfg::kBufs]);
          umma_commit(&k_empty[st]);
          return true;
        };
        ok = mbar_wait(q_full, 0, abort_flag, kKernelAttention, 75);
        for (int j = 0; j < 2 && j < n && ok; ++j) ok = issue_s(j);
        for (int j = 0; j + 2 < n && ok; ++j) {
          // Buffer (j + 2) mod 3 held P(j-1): P(j) published means O += P(j-1) V completed (the
          // softmax waits for it before storing P(j)).
          ok = mbar_wait(&p_full[j % Cfg::kBufs], (j / Cfg::kBufs) & 1, abort_flag, kKernelAttention, 79) &&
               issue_s(j + 2);
        }
      } else {
        constexpr uint32_t idesc_o = make_idesc_bf16_f32(128, HD, 0, 1);
        const uint32_t d_o = tmem_base + Cfg::kOCol;
        // O += P(j) V_j: A = P from tensor memory (16 keys = 8 packed columns per step), B = V_j
        // (MN-major: 64-wide swizzle atoms of head dims one box apart; 16 keys = 2048 bytes per step).
        for (int j = 0; j < n && ok; ++j) {
          const int st = j % Cfg::kStages;
          const int buf = j % Cfg::kBufs;
          if (!mbar_wait(&p_full[buf], (j / Cfg::kBufs) & 1, abort_flag, kKernelAttention, 73) ||
              !mbar_wait(&v_full[st], (j / Cfg::kStages) & 1, abort_flag, kKernelAttention, 74)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t v_addr = smem_u32(s_v + st * Cfg::kTileBytes);
          const uint32_t a_p = tmem_base + buf * 128;
#pragma unroll
          for (int kk = 0; kk < 128 / 16; ++kk)
            umma_bf16_ts(d_o, a_p + kk * 8, make_sdesc_sw128(v_addr + kk * 2048, Cfg::kBoxBytes, 1024), idesc_o,
                         (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(o_full);
          umma_commit(&v_empty[st]);
        }
      }
      // Both issuers commit; the barrier completes once every MMA of the CTA has.
      umma_commit(drain);
      const uint64_t t0 = global_timer_ns();
      const uint64_t lim = wait_limit_ns();
      while (!mbar_try_wait(drain, 0) && global_timer_ns() - t0 < lim) {
      }
    }
  } else {
    // ---------------- softmax ----------------
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int query = qt * 128 + r;
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t t_o = t_lane + Cfg::kOCol;
    const float c = p.scale_log2;
    const int limit = p.causal ? min(kv_len, query + 1) : kv_len;
    constexpr float kRescaleThreshold = 8.0f;  // exp2 units: rescale only when m grows by > 2^8

    float m_ref = 0.f;  // reference maximum (raw score units) used in exp2(c * (s - m_ref))
    float l_sum = 0.f;  // running sum of exp2(c * (s - m_ref)) over the row's keys (fp32)
    bool alive = true;

#pragma unroll 1
    for (int j = 0; j < n; ++j) {
      const bool last = j == n - 1;
      const int n_valid = limit - j * 128;  // keys [0, n_valid) of the last tile are visible
      const int buf = j % Cfg::kBufs;
      const uint32_t t_s = t_lane + buf * 128;
      float alpha = 1.f;
      softmax_wait(&s_full[buf], (j / Cfg::kBufs) & 1, 76, alive, abort_flag);
      tc_fence_after_sync();
      float v[128];
      tmem_load_128cols(t_s, v);
      if (last) {
#pragma unroll
        for (int k = 0; k < 128; ++k) v[k] = (k < n_valid) ? v[k] : -INFINITY;
      }
      const float rmax = fmaxf(fmaxf(max32(v), max32(v + 32)), fmaxf(max32(v + 64), max32(v + 96)));
      if (j == 0) {
        m_ref = rmax == -INFINITY ? 0.f : rmax;
      } else if ((rmax - m_ref) * c > kRescaleThreshold) {
        alpha = fast_exp2((m_ref - rmax) * c);
        m_ref = rmax;
      }
      const uint64_t c2 = splat2(c);
      const uint64_t neg_mc2 = splat2(-m_ref * c);
      // The exponentials go to registers (bf16 pairs) while O += P(j-1) V may still be running;
      // each pair of scores is dead once packed, so the live set never exceeds the 128 scores. Row
      // sums of the even and odd keys in the two halves of one packed add.
      uint64_t sum2 = 0;
      uint32_t w[64];
#pragma unroll
      for (int k = 0; k < 64; ++k) {
        float x0 = v[2 * k], x1 = v[2 * k + 1];
        fma2_inplace(x0, x1, c2, neg_mc2);
        float e0, e1;
        if ((Cfg::kPolyPairs >> (k & 3)) & 1) {
          exp2_poly_x2(x0, x1, e0, e1);
        } else {
          e0 = fast_exp2(x0);
          e1 = fast_exp2(x1);
        }
        sum2 = add2f(sum2, pack2f(e0, e1));
        w[k] = pack_bf16x2(e0, e1);
      }
      float sum0, sum1;
      unpack2f(sum2, sum0, sum1);
      l_sum = l_sum * alpha + (sum0 + sum1);
      // O += P(j-1) V must have completed before O is rescaled, and before P(j) is published: the
      // issuer reuses buffer (j + 2) mod 3, which held P(j-1), once P(j) is published.
      if (j > 0) {
        softmax_wait(o_full, (j - 1) & 1, 77, alive, abort_flag);
        tc_fence_after_sync();
      }
#pragma unroll
      for (int g = 0; g < 4; ++g) tmem_store_16cols_async(t_s + 16 * g, w + 16 * g);
      tmem_wait_st();
      if (__any_sync(0xffffffffu, alpha < 1.f)) {
        // Warp-uniform: the TMEM loads and stores are warp-collective.
#pragma unroll 1
        for (int cc = 0; cc < HD / 32; ++cc) {
          float o[32];
          tmem_load_32cols(t_o + cc * 32, o);
#pragma unroll
          for (int k = 0; k < 32; ++k) o[k] *= alpha;
          tmem_store_32cols(t_o + cc * 32, o);
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[buf]);
    }

    softmax_wait(o_full, (n - 1) & 1, 78, alive, abort_flag);
    tc_fence_after_sync();
    const float inv = l_sum > 0.f ? 1.0f / l_sum : 0.f;
    uint4* dst = reinterpret_cast<uint4*>(p.ctx + static_cast<int64_t>(row_base + query) * p.ld_ctx + h * HD);
#pragma unroll
    for (int cc = 0; cc < HD / 32; ++cc) {
      float o[32];
      tmem_load_32cols(t_o + 32 * cc, o);
      if (query < q_end) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
          dst[4 * cc + k] = make_uint4(pack_bf16x2(o[8 * k] * inv, o[8 * k + 1] * inv),
                                       pack_bf16x2(o[8 * k + 2] * inv, o[8 * k + 3] * inv),
                                       pack_bf16x2(o[8 * k + 4] * inv, o[8 * k + 5] * inv),
                                       pack_bf16x2(o[8 * k + 6] * inv, o[8 * k + 7] * inv));
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

static cudaError_t launch_attention_wide(const CUtensorMap& tm, const AttnParams& p, cudaStream_t stream) {
  using Cfg = AttnWideCfg;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(attention_wide_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    Cfg::kSmemBytes);
  });
  if (attr_err != cudaSuccess) return attr_err;
  const dim3 grid = attn_grid(p, static_cast<unsigned>(p.n_q_tiles[0] + (p.n_ranges > 1 ? p.n_q_tiles[1] : 0)));
  return launch_pdl(attention_wide_kernel, grid, dim3(Cfg::kThreads), Cfg::kSmemBytes, stream, tm, p);
}

}  // namespace b2
