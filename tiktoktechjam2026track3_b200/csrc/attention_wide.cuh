// Flash attention forward, head_dim 128, one query tile per CTA with three score buffers (the
// paths of BaselineSelfAttention.forward, transformer_benchmark/models.py:55-75; masks as in
// attention.cuh).
//
// At head_dim 128 a 128 x 128 score tile costs as many tensor-core cycles for S = Q K^T as for
// O += P V (2 x 4.2 MFLOP) and about 1000 cycles of exponentials. A kernel with two query tiles
// per CTA and one score buffer per tile (P written over it) made S(j+1) of a tile wait for
// O += P(j) V, and its tensor pipe was idle more than half the time (41.5 % active at B=1
// S=8192). Here one query tile owns three score buffers in tensor memory (3 x 128 columns, P(j)
// written over S(j)'s first 64 once the scores are in registers) and O (128 columns).
//
//   warp 0      TMA: Q once (two 64-column boxes); K_j (3-stage ring) and V_j (2-stage ring),
//               128 keys x 128 dims in two boxes each.
//   warp 1      TMEM allocator and issuer of S: S(0), S(1), S(2), then S(j) into buffer j mod 3
//               once O += P(j-3) V, the last reader of that buffer, has completed (o_done).
//   warps 2..9  softmax: the two warps of a TMEM lane quadrant share its 32 rows, 64 keys of each
//               score tile apiece (row maxima exchanged through shared memory every tile; row sums
//               added at the end): row maximum, exp2(c s - c m) as bf16 pairs (one pair in four on
//               the FMA pipe, exp2_poly_x2) into P, and, only when the reference maximum moved by
//               more than 2^8, a wait for O += P(j-1) V and the rescale of O. Without that wait the
//               softmax runs up to two tiles ahead of the tensor core.
//   warp 10     issuer of O += P(j) V_j once P(j) is published; each completion is committed to the
//               barrier of the buffer P(j) occupied (o_done).
// S and P V have separate issuers because one thread's back-to-back tcgen05.mma take at least
// ~114 clocks each at N <= 128 (measured on B200), which left the tensor core idle between the
// instructions of each product. Tensor memory (512 columns): S_b at 128 b (b = j mod 3) with P_b
// over its first 64 columns, O at 384. One CTA per SM (197 KB of shared memory).
//
// Measured on one B200 (CUDA events, L2 flushed), C4's shape (B=1, S=32768, 16 heads, causal):
// two-tile kernel 4425 us; three score buffers, one issuer 4109 us (bit-identical); one pair in
// four of the exponentials on the FMA pipe 4077 us (one in two was slower); two issuers 3861 us
// (bit-identical; boxes differ by a few percent, the steps below are same-box pairs); the softmax
// waiting for O += P(j-1) V only to rescale 3906 -> 3828 us (bit-identical); two softmax warps per
// row quadrant 3814 -> 3727 us (slower, 4115 us, while one thread issued both products).
#pragma once
#include "b2_common.cuh"
#include "attention.cuh"

namespace b2 {

struct AttnWideCfg {
  static constexpr int kSoftmaxWarps = 8;           // two per TMEM lane quadrant: 64 keys of a row each
  static constexpr int kPvWarp = 2 + kSoftmaxWarps;  // O += P V issuer (warps 2..9 are the softmax)
  static constexpr int kThreads = 32 * (kPvWarp + 1);
  static constexpr int kBoxBytes = 128 * 128;     // 128 rows x 64 bf16 columns (one TMA box)
  static constexpr int kTileBytes = 2 * kBoxBytes;  // 128 rows x 128 bf16 columns
  static constexpr int kStages = 3;               // K ring (K_j is needed two tiles before V_j)
  static constexpr int kVStages = 2;              // V ring
  static constexpr int kBufs = 3;                 // score buffers in tensor memory
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kTileBytes;
  static constexpr int kOffV = kOffK + kStages * kTileBytes;
  // Row-maximum exchange between the two warps of a row (two tiles' slots) and the final row sums.
  static constexpr int kOffRed = kOffV + kVStages * kTileBytes;
  static constexpr int kOffBar = kOffRed + 3 * 2 * 128 * 4;
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
  uint64_t* v_full = k_empty + Cfg::kStages;   // [kVStages]
  uint64_t* v_empty = v_full + Cfg::kVStages;  // [kVStages]
  uint64_t* s_full = v_empty + Cfg::kVStages;  // [kBufs]
  uint64_t* p_full = s_full + Cfg::kBufs;      // [kBufs]
  uint64_t* o_done = p_full + Cfg::kBufs;      // [kBufs]: O += P(j) V of buffer j mod 3 completed
  uint64_t* drain = o_done + Cfg::kBufs;
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
    }
    for (int i = 0; i < Cfg::kVStages; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < Cfg::kBufs; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], Cfg::kSoftmaxWarps);
      mbar_init(&o_done[i], 1);
    }
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
        if (v_next < n && mbar_test_wait(&v_empty[v_next % Cfg::kVStages], ((v_next / Cfg::kVStages) & 1) ^ 1u)) {
          const int st = v_next % Cfg::kVStages;
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
        for (int j = v_next - 1; j >= 0 && j >= v_next - Cfg::kVStages; --j)
          drain_wait(&v_full[j % Cfg::kVStages], (j / Cfg::kVStages) & 1);
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
        for (int j = 0; j < n && ok; ++j) {
          // Buffer j mod 3 held P(j-3): O += P(j-3) V must have completed (its o_done phase; the
          // buffer's next product, O += P(j) V, needs S(j), so that phase is never overtaken).
          if (j >= Cfg::kBufs)
            ok = mbar_wait(&o_done[j % Cfg::kBufs], ((j / Cfg::kBufs) - 1) & 1, abort_flag, kKernelAttention, 79);
          ok = ok && issue_s(j);
        }
      } else {
        constexpr uint32_t idesc_o = make_idesc_bf16_f32(128, HD, 0, 1);
        const uint32_t d_o = tmem_base + Cfg::kOCol;
        // O += P(j) V_j: A = P from tensor memory (16 keys = 8 packed columns per step), B = V_j
        // (MN-major: 64-wide swizzle atoms of head dims one box apart; 16 keys = 2048 bytes per step).
        for (int j = 0; j < n && ok; ++j) {
          const int st = j % Cfg::kVStages;
          const int buf = j % Cfg::kBufs;
          if (!mbar_wait(&p_full[buf], (j / Cfg::kBufs) & 1, abort_flag, kKernelAttention, 73) ||
              !mbar_wait(&v_full[st], (j / Cfg::kVStages) & 1, abort_flag, kKernelAttention, 74)) {
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
          umma_commit(&o_done[buf]);
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
    // Warps 2..9: the two warps of a TMEM lane quadrant (w and w + 4) share its 32 rows, each
    // taking 64 of a score tile's 128 keys and 64 of O's 128 head dims; per tile they exchange
    // their row maxima through shared memory (named barrier 1 + quadrant, 64 threads), so both
    // apply the same reference maximum, and they add their row sums at the end.
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quad * 32 + lane;
    const int query = qt * 128 + r;
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t t_o = t_lane + Cfg::kOCol + 64 * half;
    float* red = reinterpret_cast<float*>(smem + Cfg::kOffRed);  // [3][2][128]
    const uint32_t pair_bar = 1 + quad;
    const float c = p.scale_log2;
    const int limit = p.causal ? min(kv_len, query + 1) : kv_len;
    constexpr float kRescaleThreshold = 8.0f;  // exp2 units: rescale only when m grows by > 2^8

    float m_ref = 0.f;  // reference maximum (raw score units) used in exp2(c * (s - m_ref))
    float l_sum = 0.f;  // running sum of exp2(c * (s - m_ref)) over this warp's 64 keys of each tile
    bool alive = true;

#pragma unroll 1
    for (int j = 0; j < n; ++j) {
      const bool last = j == n - 1;
      const int n_valid = limit - j * 128 - 64 * half;  // of this warp's 64 keys, [0, n_valid) are visible
      const int buf = j % Cfg::kBufs;
      const uint32_t t_s = t_lane + buf * 128;
      float alpha = 1.f;
      softmax_wait(&s_full[buf], (j / Cfg::kBufs) & 1, 76, alive, abort_flag);
      tc_fence_after_sync();
      float v[64];
      tmem_load_64cols(t_s + 64 * half, v);
      if (last) {
#pragma unroll
        for (int k = 0; k < 64; ++k) v[k] = (k < n_valid) ? v[k] : -INFINITY;
      }
      // Row maximum over both halves (slots alternate by tile, so a slot is rewritten only after
      // the partner has passed the next exchange). After this barrier both warps have loaded their
      // scores, so P may be written over the buffer's first 64 columns.
      float* slot = red + (j & 1) * 256;
      slot[half * 128 + r] = fmaxf(max32(v), max32(v + 32));
      named_barrier_sync(pair_bar, 64);
      const float rmax = fmaxf(slot[r], slot[128 + r]);
      if (j == 0) {
        m_ref = rmax == -INFINITY ? 0.f : rmax;
      } else if ((rmax - m_ref) * c > kRescaleThreshold) {
        alpha = fast_exp2((m_ref - rmax) * c);
        m_ref = rmax;
      }
      const uint64_t c2 = splat2(c);
      const uint64_t neg_mc2 = splat2(-m_ref * c);
      // Row sums of the even and odd keys in the two halves of one packed add.
      uint64_t sum2 = 0;
      uint32_t w[32];
#pragma unroll
      for (int k = 0; k < 32; ++k) {
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
      // P(j) (this warp's 64 keys in 32 packed columns) over S(j)'s first 64 columns: both warps'
      // scores are in registers (exchange above), and the buffer's previous P, P(j-3), was
      // consumed before S(j) was issued. No wait for O += P(j-1) V unless O is rescaled, so the
      // softmax can run up to two tiles ahead of the tensor core.
#pragma unroll
      for (int g = 0; g < 2; ++g) tmem_store_16cols_async(t_s + 32 * half + 16 * g, w + 16 * g);
      tmem_wait_st();
      if (__any_sync(0xffffffffu, alpha < 1.f)) {
        // O must hold P(0..j-1) V completely (j > 0 here: alpha < 1 needs an earlier maximum); O +=
        // P(j) V is not issued before both warps of the row publish P(j). This warp's 64 columns
        // of O; warp-uniform (the TMEM loads and stores are warp-collective).
        const int jp = j - 1;
        softmax_wait(&o_done[jp % Cfg::kBufs], (jp / Cfg::kBufs) & 1, 77, alive, abort_flag);
        tc_fence_after_sync();
#pragma unroll 1
        for (int cc = 0; cc < 2; ++cc) {
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

    red[2 * 256 + half * 128 + r] = l_sum;
    named_barrier_sync(pair_bar, 64);
    const float l_row = l_sum + red[2 * 256 + (1 - half) * 128 + r];
    // O += P(n-1) V completed (the issuer's commits track all its earlier products too).
    softmax_wait(&o_done[(n - 1) % Cfg::kBufs], ((n - 1) / Cfg::kBufs) & 1, 78, alive, abort_flag);
    tc_fence_after_sync();
    const float inv = l_row > 0.f ? 1.0f / l_row : 0.f;
    uint4* dst =
        reinterpret_cast<uint4*>(p.ctx + static_cast<int64_t>(row_base + query) * p.ld_ctx + h * HD + 64 * half);
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
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
