// Flash attention forward (head_dim 64 and 128) with two query tiles per CTA (the paths of
// BaselineSelfAttention.forward, transformer_benchmark/models.py:55-75; masks as in
// attention.cuh).
//
// Why two query tiles per CTA: a 128x128 score tile costs the tensor core 2 x 128x128xhd MACs
// (S = Q K^T and O = P V: ~512 clocks at hd 64, ~1024 at hd 128) and the exponential unit 16384
// ex2 (~1024 clocks at 16/clk/SM), so at head_dim 64 the softmax, not the MMA, sets the pace and
// at 128 the two are even. With one query tile per CTA every softmax warp waits through the same
// latency phases (TMEM loads, row maximum, wait for the next S) at the same time and the
// exponential unit idles. Here each CTA owns query tiles 2c and 2c+1 with two independent 4-warp
// softmax groups; each thread owns one whole query row (no exchange between warps), so one
// group's exponentials run while the other group waits, and the tensor core alternates between
// the groups.
//
// CTA = (b, h, query-tile pair c), 12 warps at head_dim 64, 11 at head_dim 128 (or, where that
// fills the SMs better, one query tile per CTA with group 1 idle; attention_pair_tiles_per_cta):
//   warp 0      TMA: Q tiles 2c, 2c+1 once; K_j and V_j (128 keys) into two independent 4-stage
//               rings, each refilled as soon as its own slot frees (K never waits behind V).
//   warps 1, 2  UMMA issuers, one per softmax group (warp 1 also allocates TMEM). tcgen05.mma
//               issue blocks the issuing thread for about the instruction's execution time, so a
//               single issuer serving both groups would make one group's P V delay the other's
//               next S. Issuer t: S_t(j) = Q_t K_j^T into TMEM score buffer t, issued as soon as
//               group t has S_t(j-1) in registers (s_free_t); O_t += P_t(j) V_j accumulated in
//               TMEM output buffer t once P_t(j) is published (p_full_t), with P_t read straight
//               from tensor memory (A operand in TMEM) and V_j from shared memory. A K/V slot is
//               refilled after both issuers released it (a group with fewer tiles releases the
//               rest once each slot's previous use is done).
//   warp 3      (head_dim 64) spare, keeping the control warpgroup whole for the register split.
//   next 8      softmax group 0 (query tile 2c: warps 3..6 at head_dim 128, 4..7 at 64), then
//               group 1 (tile 2c+1); warp % 4 is the
//               TMEM lane quadrant = 32 query rows. Per KV tile a thread loads its row's 128 scores
//               from TMEM, takes the row maximum, writes exp2(c*s - c*m) as bf16 pairs into P_t
//               in tensor memory (tcgen05.st; lane = query row, column i = keys 2i, 2i+1) once
//               P_t(j-1) V has been accumulated (o_full_t), adds the fp32 values to its running
//               row sum, and signals p_full_t. The reference maximum m of a row only moves when
//               the tile maximum exceeds it by more than 2^8 in exp2 units (probabilities up to
//               256 are exact enough in bf16/fp32); then, and only then, the warp waits for the
//               previous accumulation and rescales its O_t rows in TMEM (and its row sum).
//
// Tensor memory: S_0, S_1 (128 columns each), P_0, P_1 (64), O_0, O_1 (64) = 512 columns.
// Shared memory traffic per tile is Q, K (S MMA) and V (P V MMA) only; P never leaves TMEM.
#pragma once
#include "b2_common.cuh"

namespace b2 {

template <int HD>
struct AttnPairCfg {
  // head_dim 64 (exponential-bound; used for launches long enough to run at the power cap): 3
  // warpgroups — control (TMA, two UMMA issuers, a spare warp), softmax group 0, group 1 — with the
  // launch's 384 x 168 registers split as control 72, softmax 216 (128 x 72 + 256 x 216 = 64512).
  // head_dim 128 (MMA and exponentials even): 11 warps, uniform 168 registers, all exponentials
  // on the exponential unit. Measured on B200: each choice is the faster one for its head_dim.
  static constexpr bool kSplitRegs = HD == 64;
  static constexpr int kThreads = kSplitRegs ? 384 : 352;
  static constexpr int kSoftmaxWarp0 = kSplitRegs ? 4 : 3;
  static constexpr int kLaunchRegs = 168;
  static constexpr int kCtrlRegs = 72;
  static constexpr int kSoftmaxRegs = 216;
  // bit k: pair k of every 4 on the FMA pipe. 0 everywhere: the head_dim-64 one-tile kernel
  // (attention_solo.cuh) takes every exponential on the exponential unit, and both head_dim-64
  // kernels must give the same bits, whichever the launch size selects.
  static constexpr int kPolyPairs = 0x0;
  static constexpr int kBoxBytes = 128 * 128;          // 128 rows x 64 bf16 columns (one TMA box)
  static constexpr int kBoxes = HD / 64;               // boxes per 128-row tile
  static constexpr int kQBytes = kBoxes * kBoxBytes;   // one 128 x HD query tile
  static constexpr int kKBytes = kQBytes;
  static constexpr int kVBytes = kQBytes;
  static constexpr int kStages = HD == 64 ? 4 : 2;
  static constexpr int kOffQ = 0;                                   // [2]
  static constexpr int kOffK = kOffQ + 2 * kQBytes;                 // [kStages]
  static constexpr int kOffV = kOffK + kStages * kKBytes;           // [kStages]
  static constexpr int kOffBar = kOffV + kStages * kVBytes;
  static constexpr int kSmemBytes = kOffBar + 256 + 1024;
  // Tensor memory (512 columns x 128 lanes of 32 bits): scores, probabilities, outputs.
  //   head_dim 64:  S_t at t * 128, P_t (128 bf16 keys packed in 64 columns) at 256 + t * 64,
  //                 O_t (64 columns) at 384 + t * 64.
  //   head_dim 128: S_t at t * 128 with P_t written over its first 64 columns (the scores are
  //                 in registers by then), O_t (128 columns) at 256 + t * 128. S_t(j+1) is issued
  //                 only after P_t(j) V has completed.
  static constexpr bool kPAliasS = HD == 128;
  static constexpr int kTmemCols = 512;
  static constexpr int kSCol = 0;
  static constexpr int kPCol = kPAliasS ? 0 : 256;
  static constexpr int kPStride = kPAliasS ? 128 : 64;
  static constexpr int kOCol = kPAliasS ? 256 : 384;
  static_assert(kSmemBytes <= 232448, "shared memory per CTA");
};

// Row maximum of 32 values as a balanced tree of 3-input maxima (short dependency chains).
__device__ __forceinline__ float max32(const float* v) {
  float a[11];
#pragma unroll
  for (int i = 0; i < 10; ++i) a[i] = max3f(v[3 * i], v[3 * i + 1], v[3 * i + 2]);
  a[10] = fmaxf(v[30], v[31]);
  const float b0 = max3f(a[0], a[1], a[2]);
  const float b1 = max3f(a[3], a[4], a[5]);
  const float b2 = max3f(a[6], a[7], a[8]);
  const float b3 = fmaxf(a[9], a[10]);
  return fmaxf(max3f(b0, b1, b2), b3);
}

template <int HD>
__global__ void __launch_bounds__(AttnPairCfg<HD>::kThreads, 1)
    attention_pair_kernel(const __grid_constant__ CUtensorMap tm_qkv, const AttnParams p) {
  using Cfg = AttnPairCfg<HD>;
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
  uint64_t* s_full = v_empty + Cfg::kStages;   // [2 groups]
  uint64_t* p_full = s_full + 2;               // [2 groups]
  uint64_t* o_full = p_full + 2;               // [2 groups]
  uint64_t* s_free = o_full + 2;               // [2 groups]
  uint64_t* drain = s_free + 2;                // [2 issuers]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int bh, cta_row;
  attn_cta_coords(p, bh, cta_row);
  const int b = bh / p.H;
  const int h = bh % p.H;
  const int tpc = p.tiles_per_cta;  // query tiles per CTA: 2, or 1 with group 1 idle
  const int range_pairs[2] = {(p.n_q_tiles[0] + tpc - 1) / tpc, (p.n_q_tiles[1] + tpc - 1) / tpc};
  int y_local;
  const int rg = attn_range_of(p, cta_row, range_pairs, y_local);
  const int pair = range_pairs[rg] - 1 - y_local;  // heaviest causal pairs first
  const int q_tile0 = p.q_tile0[rg];
  const int q_end = p.q_end[rg];
  const int kv_len = p.kv_len != nullptr ? p.kv_len[b] : p.S;
  const int kv_tiles = (kv_len + 127) >> 7;
  int n_kv[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int qt = q_tile0 + tpc * pair + t;  // absolute query tile
    const bool live = t < tpc && tpc * pair + t < p.n_q_tiles[rg] && qt * 128 < kv_len;
    n_kv[t] = live ? (p.causal ? min(qt + 1, kv_tiles) : kv_tiles) : 0;
  }
  const int n_total = max(n_kv[0], n_kv[1]);
  if (n_total == 0) return;  // uniform for the CTA: nothing allocated yet
  const int row_base = b * p.S;
  const int q_row0 = row_base + (q_tile0 + tpc * pair) * 128;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < Cfg::kStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 2);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 2);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_full[i], 1);
      mbar_init(&s_free[i], 4);
    }
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
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
  static_assert(!Cfg::kSplitRegs || 128 * Cfg::kCtrlRegs + 256 * Cfg::kSoftmaxRegs <= Cfg::kThreads * Cfg::kLaunchRegs,
                "register split");

  if (warp < Cfg::kSoftmaxWarp0) {
   if constexpr (Cfg::kSplitRegs) regs_dec<Cfg::kCtrlRegs>();
   if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const int qc = p.q_col + h * HD;
      const int kc = p.k_col + h * HD;
      const int vc = p.v_col + h * HD;
      mbar_arrive_expect_tx(q_full, static_cast<uint32_t>(tpc * Cfg::kQBytes));
#pragma unroll
      for (int c = 0; c < Cfg::kBoxes; ++c) {
        tma_load_2d(s_q + c * Cfg::kBoxBytes, &tm_qkv, q_full, qc + 64 * c, q_row0);
        if (tpc == 2)
          tma_load_2d(s_q + Cfg::kQBytes + c * Cfg::kBoxBytes, &tm_qkv, q_full, qc + 64 * c, q_row0 + 128);
      }
      // K and V rings refill independently (polling both), so a K tile never waits for a V slot.
      int k_next = 0, v_next = 0;
      bool ok = true;
      PollTimeout poll;
      poll.reset();
      while (k_next < n_total || v_next < n_total) {
        bool progress = false;
        if (k_next < n_total &&
            mbar_test_wait(&k_empty[k_next % Cfg::kStages], ((k_next / Cfg::kStages) & 1) ^ 1u)) {
          const int st = k_next % Cfg::kStages;
          mbar_arrive_expect_tx(&k_full[st], Cfg::kKBytes);
#pragma unroll
          for (int c = 0; c < Cfg::kBoxes; ++c)
            tma_load_2d(s_k + st * Cfg::kKBytes + c * Cfg::kBoxBytes, &tm_qkv, &k_full[st], kc + 64 * c,
                        row_base + k_next * 128);
          ++k_next;
          progress = true;
        }
        if (v_next < n_total &&
            mbar_test_wait(&v_empty[v_next % Cfg::kStages], ((v_next / Cfg::kStages) & 1) ^ 1u)) {
          const int st = v_next % Cfg::kStages;
          mbar_arrive_expect_tx(&v_full[st], Cfg::kVBytes);
#pragma unroll
          for (int c = 0; c < Cfg::kBoxes; ++c)
            tma_load_2d(s_v + st * Cfg::kVBytes + c * Cfg::kBoxBytes, &tm_qkv, &v_full[st], vc + 64 * c,
                        row_base + v_next * 128);
          ++v_next;
          progress = true;
        }
        if (progress) {
          poll.reset();
        } else if (*abort_flag) {
          ok = false;
          break;
        } else if (poll.expired()) {
          record_status(kKernelAttention, 21, kReasonTimeout);
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
  } else if (warp == 1 || warp == 2) {
    // ---------------- UMMA issuers (one per group) ----------------
    const int t = warp - 1;
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16_f32(128, 128, 0, 0);
      constexpr uint32_t idesc_o = make_idesc_bf16_f32(128, HD, 0, 1);
      const uint32_t q_addr = smem_u32(s_q) + t * Cfg::kQBytes;
      const uint32_t d_s = tmem_base + Cfg::kSCol + t * 128;
      const uint32_t d_o = tmem_base + Cfg::kOCol + t * HD;
      const uint32_t a_p = tmem_base + Cfg::kPCol + t * Cfg::kPStride;
      const int n = n_kv[t];
      auto issue_s = [&](int j) {
        const uint32_t k_addr = smem_u32(s_k + (j % Cfg::kStages) * Cfg::kKBytes);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * Cfg::kBoxBytes + (kk & 3) * 32;
          umma_bf16_ss(d_s, make_sdesc_sw128(q_addr + off, 16, 1024), make_sdesc_sw128(k_addr + off, 16, 1024),
                       idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
        umma_commit(&k_empty[j % Cfg::kStages]);
      };
      auto issue_o = [&](int j) {
        const int vst = j % Cfg::kStages;
        const uint32_t v_addr = smem_u32(s_v + vst * Cfg::kVBytes);
        // A = P_t from tensor memory (16 keys = 8 packed columns per step), B = V_j (MN-major:
        // 64-wide swizzle atoms of head dims, one box apart; 16 keys = 2048 bytes per step).
#pragma unroll
        for (int kk = 0; kk < 128 / 16; ++kk)
          umma_bf16_ts(d_o, a_p + kk * 8, make_sdesc_sw128(v_addr + kk * 2048, Cfg::kBoxBytes, 1024), idesc_o,
                       (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&o_full[t]);
        umma_commit(&v_empty[vst]);
      };
      bool ok = n == 0 || mbar_wait(q_full, 0, abort_flag, kKernelAttention, 23);
      for (int j = 0; j < n && ok; ++j) {
        // S_t(j): K_j loaded and (j > 0) S_t(j-1) taken by the softmax group; with P_t stored
        // over S_t, also P_t(j-1) V complete.
        if (!mbar_wait(&k_full[j % Cfg::kStages], (j / Cfg::kStages) & 1, abort_flag, kKernelAttention, 24) ||
            (j > 0 && !mbar_wait(&s_free[t], (j - 1) & 1, abort_flag, kKernelAttention, 25)) ||
            (Cfg::kPAliasS && j > 0 && !mbar_wait(&o_full[t], (j - 1) & 1, abort_flag, kKernelAttention, 33))) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        issue_s(j);
        if (Cfg::kPAliasS) {
          // O_t += P_t(j) V_j as soon as published: S_t(j + 1) waits for it anyway.
          if (!mbar_wait(&p_full[t], j & 1, abort_flag, kKernelAttention, 26) ||
              !mbar_wait(&v_full[j % Cfg::kStages], (j / Cfg::kStages) & 1, abort_flag, kKernelAttention, 27)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          issue_o(j);
          continue;
        }
        // O_t += P_t(j-1) V_{j-1} once published (issued after S_t(j) so the scores come first).
        if (j > 0) {
          if (!mbar_wait(&p_full[t], (j - 1) & 1, abort_flag, kKernelAttention, 26) ||
              !mbar_wait(&v_full[(j - 1) % Cfg::kStages], ((j - 1) / Cfg::kStages) & 1, abort_flag,
                         kKernelAttention, 27)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          issue_o(j - 1);
        }
      }
      if (ok && n > 0 && !Cfg::kPAliasS) {
        if (!mbar_wait(&p_full[t], (n - 1) & 1, abort_flag, kKernelAttention, 26) ||
            !mbar_wait(&v_full[(n - 1) % Cfg::kStages], ((n - 1) / Cfg::kStages) & 1, abort_flag, kKernelAttention,
                       27)) {
          ok = false;
        } else {
          tc_fence_after_sync();
          issue_o(n - 1);
        }
      }
      // K/V tiles this group does not use: release each slot for the producer once its previous
      // use is over (a plain arrive here would otherwise count toward the previous phase).
      for (int j = n; j < n_total && ok; ++j) {
        const int st = j % Cfg::kStages;
        const uint32_t prev = ((j / Cfg::kStages) & 1) ^ 1u;
        if (!mbar_wait(&k_empty[st], prev, abort_flag, kKernelAttention, 31) ||
            !mbar_wait(&v_empty[st], prev, abort_flag, kKernelAttention, 32)) {
          ok = false;
          break;
        }
        mbar_arrive(&k_empty[st]);
        mbar_arrive(&v_empty[st]);
      }
      umma_commit(&drain[t]);
      const uint64_t t0 = global_timer_ns();
      const uint64_t lim = wait_limit_ns();
      while (!mbar_try_wait(&drain[t], 0) && global_timer_ns() - t0 < lim) {
      }
    }
   }
  } else {
    if constexpr (Cfg::kSplitRegs) regs_inc<Cfg::kSoftmaxRegs>();
    // ---------------- softmax groups ----------------
    const int grp = (warp - Cfg::kSoftmaxWarp0) >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int qt = q_tile0 + tpc * pair + grp;
    const int query = qt * 128 + r;
    const int n = grp == 0 ? n_kv[0] : n_kv[1];
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t t_s = t_lane + Cfg::kSCol + grp * 128;
    const uint32_t t_o = t_lane + Cfg::kOCol + grp * HD;
    const uint32_t t_p = t_lane + Cfg::kPCol + grp * Cfg::kPStride;
    const float c = p.scale_log2;
    const int limit = p.causal ? min(kv_len, query + 1) : kv_len;
    constexpr float kRescaleThreshold = 8.0f;  // exp2 units: rescale only when m grows by > 2^8
    constexpr int kPolyPairs = Cfg::kPolyPairs;

    float m_ref = 0.f;  // reference maximum (raw score units) used in exp2(c * (s - m_ref))
    float l_sum = 0.f;  // running sum of exp2(c * (s - m_ref)) over the row's keys (fp32)
    bool alive = true;

    // Ping-pong of the exponential phase between the groups: group g runs its exp2 loop only
    // after the other group finished its previous one (named barrier 1 + g completes when the 128
    // threads of group g sync and the 128 of the other group arrive), so each SM sub-partition's
    // exponential unit (16/clk/SM) serves one group while the other loads and reduces its next
    // score tile. Both groups run n_total rounds (idle rounds only pass the barriers) so the
    // arrive/sync counts match; group 1 pre-arrives once and skips its last arrive.
    if (grp == 1) named_barrier_arrive(1, 256);

#pragma unroll 1
    for (int j = 0; j < n_total; ++j) {
      const bool work = j < n;
      const bool last = j == n - 1;
      const int n_valid = limit - j * 128;  // keys [0, n_valid) of the last tile are visible
      float alpha = 1.f;  // < 1 when this row's reference maximum moves (rare after the first tile)
      if (work) {
        // Row maximum first (scores are read again after the handoff, so none are held across it).
        softmax_wait(&s_full[grp], j & 1, 28, alive, abort_flag);
        tc_fence_after_sync();
        float rmax;
        {
          float v[128];
          tmem_load_128cols(t_s, v);
          if (last) {
#pragma unroll
            for (int k = 0; k < 128; ++k) v[k] = (k < n_valid) ? v[k] : -INFINITY;
          }
          rmax = fmaxf(fmaxf(max32(v), max32(v + 32)), fmaxf(max32(v + 64), max32(v + 96)));
        }
        if (j == 0) {
          m_ref = rmax == -INFINITY ? 0.f : rmax;
        } else if ((rmax - m_ref) * c > kRescaleThreshold) {
          alpha = fast_exp2((m_ref - rmax) * c);
          m_ref = rmax;
        }
        // P_t(j-1) V must have been accumulated before P_t is overwritten (and before a rescale).
        if (j > 0) {
          softmax_wait(&o_full[grp], (j - 1) & 1, 29, alive, abort_flag);
          tc_fence_after_sync();
        }
      }
      if (grp == 0)
        named_barrier_sync(1, 256);
      else
        named_barrier_sync(2, 256);
      if (work) {
        float v[128];
        tmem_load_128cols(t_s, v);
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[grp]);  // S_t may now receive tile j + 1
        if (last) {
#pragma unroll
          for (int k = 0; k < 128; ++k) v[k] = (k < n_valid) ? v[k] : -INFINITY;
        }
        const uint64_t c2 = splat2(c);
        const uint64_t neg_mc2 = splat2(-m_ref * c);
        // probabilities -> P_t in tensor memory: row r = lane r, keys 2i, 2i+1 packed in column i.
        // Pairs selected by kPolyPairs take 2^x on the FMA pipe (exp2_poly_x2), the others on the
        // exponential unit, so that both pipes share the 16384 exponentials of a tile.
        float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          uint32_t w[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            float x0 = v[32 * g + 2 * k], x1 = v[32 * g + 2 * k + 1];
            fma2_inplace(x0, x1, c2, neg_mc2);
            float e0, e1;
            if ((kPolyPairs >> (k & 3)) & 1) {
              exp2_poly_x2(x0, x1, e0, e1);
            } else {
              e0 = fast_exp2(x0);
              e1 = fast_exp2(x1);
            }
            sum0 += e0;
            sum1 += e1;
            w[k] = pack_bf16x2(e0, e1);
          }
          tmem_store_16cols_async(t_p + 16 * g, w);
        }
        l_sum = l_sum * alpha + (sum0 + sum1);
        tmem_wait_st();
      }
      if (grp == 0)
        named_barrier_arrive(2, 256);
      else if (j < n_total - 1)
        named_barrier_arrive(1, 256);
      if (work) {
        if (__any_sync(0xffffffffu, alpha < 1.f)) {
          // Rescale the accumulated output and row sums (P_t(0..j-1) V) of the warp's rows to their
          // new reference maxima (alpha = 1 for rows whose maximum did not move); the accumulation
          // of tile j-1 has landed (waited above) and P_t(j) V is not issued before p_full_t.
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
        if (lane == 0) mbar_arrive(&p_full[grp]);
      }
    }

    if (n > 0) {
      softmax_wait(&o_full[grp], (n - 1) & 1, 30, alive, abort_flag);
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
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

int device_sm_count(int device);

// Query tiles per CTA. Two tiles (one per softmax group) share the exponential unit and the K/V
// stream; a single-tile CTA (group 1 idle) takes about 0.75 of a pair CTA's time (measured on
// B200: C2's attention, 192 pair CTAs in two waves 37.8 us, 384 single-tile CTAs in three waves
// 42.4 us). Single-tile CTAs are chosen when their wave count times that factor beats the pair
// waves — in practice when both fit the same number of waves, so the extra CTAs fill idle SMs
// (B=1 S=1024 16 heads: 33.2 -> 29.9 us; B=2 S=512 head_dim 128: 30.2 -> 27.9 us).
static int attention_pair_tiles_per_cta(const AttnParams& p, int sms) {
  constexpr double kSingleCost = 0.75;  // single-tile CTA time / pair CTA time (same KV tiles)
  long tiles = 0, pairs = 0;
  for (int r = 0; r < p.n_ranges; ++r) {
    tiles += p.n_q_tiles[r];
    pairs += (p.n_q_tiles[r] + 1) / 2;
  }
  const long ctas2 = static_cast<long>(p.B) * p.H * pairs;
  const long ctas1 = static_cast<long>(p.B) * p.H * tiles;
  const long waves2 = (ctas2 + sms - 1) / sms;
  const long waves1 = (ctas1 + sms - 1) / sms;
  return kSingleCost * static_cast<double>(waves1) < static_cast<double>(waves2) ? 1 : 2;
}

template <int HD>
static cudaError_t launch_attention_pair(const CUtensorMap& tm, const AttnParams& p, cudaStream_t stream) {
  // Launched for head_dim 128 only; head_dim 64 runs on the one-tile kernel (attention_solo.cuh),
  // measured faster at every benchmark size. The template's head_dim-64 configuration (register
  // split, 4-stage rings) is not instantiated.
  using Cfg = AttnPairCfg<HD>;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(attention_pair_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    Cfg::kSmemBytes);
  });
  if (attr_err != cudaSuccess) return attr_err;
  AttnParams q = p;
  q.tiles_per_cta = attention_pair_tiles_per_cta(p, device_sm_count(dev));
  const int t = q.tiles_per_cta;
  const dim3 grid = attn_grid(q, static_cast<unsigned>((p.n_q_tiles[0] + t - 1) / t +
                                                       (p.n_ranges > 1 ? (p.n_q_tiles[1] + t - 1) / t : 0)));
  return launch_pdl(attention_pair_kernel<HD>, grid, dim3(Cfg::kThreads), Cfg::kSmemBytes, stream, tm, q);
}

}  // namespace b2
