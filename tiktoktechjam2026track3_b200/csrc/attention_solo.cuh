// Flash attention forward, head_dim 64, one query tile per CTA and two CTAs per SM (the paths of
// BaselineSelfAttention.forward, transformer_benchmark/models.py:55-75; masks as in attention.cuh).
//
// For short sequences the work of a layer is a few hundred query tiles of 2-4 KV tiles each
// (C2: 8 x 512 tokens, 12 heads, padded lengths in [256, 512]). A kernel with two query tiles per
// CTA (384 threads x 168 registers, 160 KB of shared memory, one CTA per SM, its two softmax
// groups alternating on the exponential unit) ran them as two waves of long-latency CTAs: a
// per-CTA trace showed each CTA spending ~2.4 us waiting for its first Q tile and ~1.7 us per KV
// tile on its chain of S = Q K^T -> row max -> exponentials -> O += P V, with the second wave
// starting only when the first had drained. This kernel is the same computation for one query
// tile with 6 warps (192 threads x 168 registers), 80 KB of shared memory (2-stage K and V rings)
// and 256 TMEM columns, so that two CTAs share an SM: their chains interleave on the tensor core
// and the exponential unit without any ping-pong between them, and a CTA of the next wave starts
// as soon as either resident CTA ends.
//
//   warp 0      TMA: Q once; K_j and V_j (128 keys) into two independent 2-stage rings.
//   warp 1      TMEM allocator and UMMA issuer: S(j) = Q K_j^T into TMEM once S(j-1) has been
//               read (s_free), then O += P(j-1) V_{j-1} once P(j-1) is published (p_full), P read
//               from TMEM as the A operand.
//   warps 2..5  softmax, one query row per thread (warp % 4 = TMEM lane quadrant): row maximum
//               from the scores in TMEM, exp2(c s - c m) computed into registers as bf16 pairs
//               and stored into P in TMEM after O += P(j-1) V has landed (o_full), fp32 row sums
//               in registers, lazy rescale (the reference maximum moves only by more than 2^8).
// Tensor memory: S (128 columns) at 0, P (128 bf16 keys in 64 columns) at 128, O (64) at 192.
// Measured on one B200 against the two-tile kernel (CUDA events, L2 flushed): C2's attention
// (B=8, S=512, 12 heads, padded) 33.3 -> 28.3 us, B=16 S=2048 causal 321 -> 254 us, B=1 S=16384
// causal 871 -> 743 us (631 -> 740 TFLOP/s): two softmax warps per SM sub-partition keep the
// exponential unit busier than the two-tile kernel's ping-pong between its groups. At C5 (4 x 100000
// tokens, ~110 ms per launch at the 1000 W power cap) with the head-major grid order it runs at
// 752 TFLOP/s against 672 for the two-tile kernel: with K/V served from L2, streaming them once
// per query tile no longer costs more than the scheduling gains. It is the head_dim-64 kernel for
// every shape. Computing the exponentials of tile j into registers before waiting for
// O += P(j-1) V (only the store into P waits) gave, with bit-identical outputs: B=16 S=2048 causal
// 247.8 -> 239.6 us, B=1 S=16384 841.7 -> 825.3 us, 4 x 100000 causal 106.8 -> 105.6 ms, head_dim
// 32 (B=64 S=1024, 4 heads) 82.0 -> 79.9 us; C2's shape unchanged.
#pragma once
#include "b2_common.cuh"
#include "attention.cuh"

namespace b2 {

struct AttnSoloCfg {
  static constexpr int kThreads = 192;
  static constexpr int kSoftmaxWarp0 = 2;
  static constexpr int kTileBytes = 128 * 128;  // 128 rows x 64 bf16 columns (one TMA box)
  static constexpr int kStages = 2;
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kTileBytes;
  static constexpr int kOffV = kOffK + kStages * kTileBytes;
  static constexpr int kOffBar = kOffV + kStages * kTileBytes;
  static constexpr int kSmemBytes = kOffBar + 256 + 1024;
  static constexpr int kTmemCols = 256;
  static constexpr int kSCol = 0;
  static constexpr int kPCol = 128;
  static constexpr int kOCol = 192;
  static_assert(2 * (kSmemBytes + 1024) <= 233472, "two CTAs per SM");
};

// HD = 64, or 32 (the reference's official case matrix: D = 128 with 4 heads). At head_dim 32 every
// tile is still loaded as a 64-column TMA box (the head's 32 columns and the next 32 of the packed
// QKV row, zero-filled past its end): S = Q K^T takes only the first two 16-deep k-steps, i.e. this
// head's columns, and O += P V is computed 64 wide, its second half (the neighbouring columns)
// discarded — the exponentials, not the MMAs, bound the kernel, and the operand layouts stay the
// 128-byte-swizzled ones of head_dim 64.
template <int HD>
__global__ void __launch_bounds__(AttnSoloCfg::kThreads, 2)
    attention_solo_kernel(const __grid_constant__ CUtensorMap tm_qkv, const AttnParams p) {
  static_assert(HD == 32 || HD == 64, "one-tile kernel: head_dim 32 or 64");
  using Cfg = AttnSoloCfg;
  constexpr int kON = 64;  // columns of O (and width of the P V product)
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
  uint64_t* s_full = v_empty + Cfg::kStages;
  uint64_t* p_full = s_full + 1;
  uint64_t* o_full = p_full + 1;
  uint64_t* s_free = o_full + 1;
  uint64_t* drain = s_free + 1;
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
    mbar_init(s_full, 1);
    mbar_init(p_full, 4);
    mbar_init(o_full, 1);
    mbar_init(s_free, 4);
    mbar_init(drain, 1);
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
      int k_next = 0, v_next = 0;
      bool ok = true;
      PollTimeout poll;
      poll.reset();
      while (k_next < n || v_next < n) {
        bool progress = false;
        if (k_next < n && mbar_test_wait(&k_empty[k_next % Cfg::kStages], ((k_next / Cfg::kStages) & 1) ^ 1u)) {
          const int st = k_next % Cfg::kStages;
          mbar_arrive_expect_tx(&k_full[st], Cfg::kTileBytes);
          tma_load_2d(s_k + st * Cfg::kTileBytes, &tm_qkv, &k_full[st], kc, row_base + k_next * 128);
          ++k_next;
          progress = true;
        }
        if (v_next < n && mbar_test_wait(&v_empty[v_next % Cfg::kStages], ((v_next / Cfg::kStages) & 1) ^ 1u)) {
          const int st = v_next % Cfg::kStages;
          mbar_arrive_expect_tx(&v_full[st], Cfg::kTileBytes);
          tma_load_2d(s_v + st * Cfg::kTileBytes, &tm_qkv, &v_full[st], vc, row_base + v_next * 128);
          ++v_next;
          progress = true;
        }
        if (progress) {
          poll.reset();
        } else if (*abort_flag) {
          ok = false;
          break;
        } else if (poll.expired()) {
          record_status(kKernelAttention, 41, kReasonTimeout);
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
  } else if (warp == 1) {
    // ---------------- UMMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16_f32(128, 128, 0, 0);
      constexpr uint32_t idesc_o = make_idesc_bf16_f32(128, kON, 0, 1);
      const uint32_t q_addr = smem_u32(s_q);
      const uint32_t d_s = tmem_base + Cfg::kSCol;
      const uint32_t d_o = tmem_base + Cfg::kOCol;
      const uint32_t a_p = tmem_base + Cfg::kPCol;
      auto issue_s = [&](int j) {
        const uint32_t k_addr = smem_u32(s_k + (j % Cfg::kStages) * Cfg::kTileBytes);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          umma_bf16_ss(d_s, make_sdesc_sw128(q_addr + kk * 32, 16, 1024), make_sdesc_sw128(k_addr + kk * 32, 16, 1024),
                       idesc_s, kk > 0 ? 1u : 0u);
        umma_commit(s_full);
        umma_commit(&k_empty[j % Cfg::kStages]);
      };
      auto issue_o = [&](int j) {
        const int vst = j % Cfg::kStages;
        const uint32_t v_addr = smem_u32(s_v + vst * Cfg::kTileBytes);
        // A = P from tensor memory (16 keys = 8 packed columns per step), B = V_j (MN-major, 16
        // keys = 2048 bytes per step).
#pragma unroll
        for (int kk = 0; kk < 128 / 16; ++kk)
          umma_bf16_ts(d_o, a_p + kk * 8, make_sdesc_sw128(v_addr + kk * 2048, Cfg::kTileBytes, 1024), idesc_o,
                       (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(o_full);
        umma_commit(&v_empty[vst]);
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, kKernelAttention, 43);
      for (int j = 0; j < n && ok; ++j) {
        if (!mbar_wait(&k_full[j % Cfg::kStages], (j / Cfg::kStages) & 1, abort_flag, kKernelAttention, 44) ||
            (j > 0 && !mbar_wait(s_free, (j - 1) & 1, abort_flag, kKernelAttention, 45))) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        issue_s(j);
        // O += P(j-1) V_{j-1} once published (issued after S(j) so the scores come first).
        if (j > 0) {
          if (!mbar_wait(p_full, (j - 1) & 1, abort_flag, kKernelAttention, 46) ||
              !mbar_wait(&v_full[(j - 1) % Cfg::kStages], ((j - 1) / Cfg::kStages) & 1, abort_flag, kKernelAttention,
                         47)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          issue_o(j - 1);
        }
      }
      if (ok) {
        if (!mbar_wait(p_full, (n - 1) & 1, abort_flag, kKernelAttention, 46) ||
            !mbar_wait(&v_full[(n - 1) % Cfg::kStages], ((n - 1) / Cfg::kStages) & 1, abort_flag, kKernelAttention,
                       47)) {
          ok = false;
        } else {
          tc_fence_after_sync();
          issue_o(n - 1);
        }
      }
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
    const uint32_t t_s = t_lane + Cfg::kSCol;
    const uint32_t t_o = t_lane + Cfg::kOCol;
    const uint32_t t_p = t_lane + Cfg::kPCol;
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
      float alpha = 1.f;
      softmax_wait(s_full, j & 1, 48, alive, abort_flag);
      tc_fence_after_sync();
      float v[128];
      tmem_load_128cols(t_s, v);
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);  // S may now receive tile j + 1
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
      // The exponentials of tile j go to registers (bf16 pairs) while O += P(j-1) V is still
      // running on the tensor core; only their store into P waits for it. Row sums of the even and
      // odd keys in the two halves of one packed add (the same per-lane rounding as two scalar
      // sums). Each pair of scores is dead once packed, so the live set never exceeds the 128
      // scores.
      uint64_t sum2 = 0;
      uint32_t w[64];
#pragma unroll
      for (int k = 0; k < 64; ++k) {
        float x0 = v[2 * k], x1 = v[2 * k + 1];
        fma2_inplace(x0, x1, c2, neg_mc2);
        const float e0 = fast_exp2(x0);
        const float e1 = fast_exp2(x1);
        sum2 = add2f(sum2, pack2f(e0, e1));
        w[k] = pack_bf16x2(e0, e1);
      }
      float sum0, sum1;
      unpack2f(sum2, sum0, sum1);
      l_sum = l_sum * alpha + (sum0 + sum1);
      // P(j-1) V must have been accumulated before P is overwritten (and before a rescale).
      if (j > 0) {
        softmax_wait(o_full, (j - 1) & 1, 49, alive, abort_flag);
        tc_fence_after_sync();
      }
#pragma unroll
      for (int g = 0; g < 4; ++g) tmem_store_16cols_async(t_p + 16 * g, w + 16 * g);
      tmem_wait_st();
      if (__any_sync(0xffffffffu, alpha < 1.f)) {
        // Rescale the accumulated output of the warp's rows (P(0..j-1) V, landed above); P(j) V is
        // not issued before p_full. Warp-uniform: the TMEM loads and stores are warp-collective.
#pragma unroll 1
        for (int cc = 0; cc < kON / 32; ++cc) {
          float o[32];
          tmem_load_32cols(t_o + cc * 32, o);
#pragma unroll
          for (int k = 0; k < 32; ++k) o[k] *= alpha;
          tmem_store_32cols(t_o + cc * 32, o);
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }

    softmax_wait(o_full, (n - 1) & 1, 50, alive, abort_flag);
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

template <int HD>
static cudaError_t launch_attention_solo(const CUtensorMap& tm, const AttnParams& p, cudaStream_t stream) {
  using Cfg = AttnSoloCfg;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(attention_solo_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    Cfg::kSmemBytes);
  });
  if (attr_err != cudaSuccess) return attr_err;
  const dim3 grid = attn_grid(p, static_cast<unsigned>(p.n_q_tiles[0] + (p.n_ranges > 1 ? p.n_q_tiles[1] : 0)));
  return launch_pdl(attention_solo_kernel<HD>, grid, dim3(Cfg::kThreads), Cfg::kSmemBytes, stream, tm, p);
}

}  // namespace b2
