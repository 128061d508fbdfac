// Flash-style multi-head self-attention forward: the shared parameters, the host entry point,
// and the softmax helpers. The tcgen05 kernels are in attention_solo.cuh (head_dim 32 and 64,
// one query tile per CTA, two CTAs per SM) and attention_wide.cuh (head_dim 128, one query tile
// per CTA with three score buffers); head dims 8, 16 and 256 run on CUDA cores (attention_simt.cuh).
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
  // Query rows computed per sequence: up to two ranges (the second one later in the sequence, so
  // its CTAs, the heavier ones under a causal mask, are issued first). Queries are absolute
  // positions for the causal mask.
  int n_ranges;
  int q_tile0[2];    // first query tile (128 rows) of the range
  int n_q_tiles[2];  // query tiles in the range
  int q_end[2];      // one past the last query row of the range
  // Grid order of the tensor-core kernels: 1 = query blocks along x and (b, h) along y, so the
  // hardware issues every query block of one head (heaviest first) before the next head and the
  // CTAs resident at any time read the K/V rows of one or two heads, which stay in L2 (a
  // 100000-token head's K and V are 25.6 MB); 0 = (b, h) along x, so the heaviest query blocks of
  // every head go first. Long sequences (S >= 16384) take 1: at B=4, S=100000 it measured 133.3 ->
  // 121.9 ms per launch (the K/V streams of the resident CTAs no longer miss L2). Short ones take 0,
  // whose K/V fit L2 either way and whose tail is shorter with the global heaviest-first order
  // (C2 28.3 vs 30.1 us, B=16 S=2048 causal 254 vs 276 us). Either order computes the same values.
  int head_major;
};

// (b, h) and the query-block row of this CTA in the grid order of AttnParams::head_major.
__device__ __forceinline__ void attn_cta_coords(const AttnParams& p, int& bh, int& row) {
  if (p.head_major) {
    bh = static_cast<int>(blockIdx.y);
    row = static_cast<int>(blockIdx.x);
  } else {
    bh = static_cast<int>(blockIdx.x);
    row = static_cast<int>(blockIdx.y);
  }
}

static inline dim3 attn_grid(const AttnParams& p, unsigned rows) {
  const unsigned bh = static_cast<unsigned>(p.B) * static_cast<unsigned>(p.H);
  return p.head_major ? dim3(rows, bh) : dim3(bh, rows);
}

// Query range of the CTA row `y` of a grid whose rows cover `per_range[r]` work items of range r,
// range 1 first.
__device__ __forceinline__ int attn_range_of(const AttnParams& p, int y, const int (&per_range)[2], int& local) {
  if (p.n_ranges > 1 && y < per_range[1]) {
    local = y;
    return 1;
  }
  local = y - (p.n_ranges > 1 ? per_range[1] : 0);
  return 0;
}

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

// Softmax-warp wait: once any wait of this thread gave up (`alive` false) later waits are
// skipped, so the warp still runs its remaining iterations and every named barrier stays matched.
__device__ __forceinline__ void softmax_wait(uint64_t* bar, uint32_t parity, uint32_t site, bool& alive,
                                             volatile int* abort_flag) {
  if (alive && !mbar_wait(bar, parity, abort_flag, kKernelAttention, site)) alive = false;
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------
cudaError_t make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                              uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer);

template <int HD>
static cudaError_t launch_attention_simt(const __nv_bfloat16* qkv, int64_t ld_qkv, const AttnParams& p,
                                         cudaStream_t stream);

template <int HD>
static cudaError_t launch_attention_solo(const CUtensorMap& tm, const AttnParams& p, cudaStream_t stream);

static cudaError_t launch_attention_wide(const CUtensorMap& tm, const AttnParams& p, cudaStream_t stream);


cudaError_t launch_attention(const __nv_bfloat16* qkv, int64_t ld_qkv, int64_t q_col, int64_t k_col, int64_t v_col,
                             int64_t B, int64_t S, int64_t H, int64_t hd, const int32_t* kv_len, int causal,
                             float scale, __nv_bfloat16* ctx, int64_t ld_ctx, cudaStream_t stream,
                             const int64_t* q_ranges = nullptr, int n_ranges = 0) {
  const int64_t whole[2] = {0, S};
  if (n_ranges == 0) {
    q_ranges = whole;
    n_ranges = 1;
  }
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
  p.n_ranges = n_ranges;
  p.head_major = (S >= 16384 && B * H <= 65535) ? 1 : 0;
  for (int r = 0; r < 2; ++r) {
    const int64_t q_begin = r < n_ranges ? q_ranges[2 * r] : 0;
    const int64_t q_count = r < n_ranges ? q_ranges[2 * r + 1] : 0;
    p.q_tile0[r] = static_cast<int>(q_begin / 128);
    p.q_end[r] = static_cast<int>(q_begin + q_count);
    p.n_q_tiles[r] = static_cast<int>((q_count + 127) / 128);
  }
  switch (hd) {
    case 8:
      return launch_attention_simt<8>(qkv, ld_qkv, p, stream);
    case 16:
      return launch_attention_simt<16>(qkv, ld_qkv, p, stream);
    case 256:
      return launch_attention_simt<256>(qkv, ld_qkv, p, stream);
    default:
      break;
  }
  if (hd != 32 && hd != 64 && hd != 128) return cudaErrorInvalidValue;
  CUtensorMap tm;
  cudaError_t e = make_tmap_bf16_2d(&tm, qkv, static_cast<uint64_t>(ld_qkv), static_cast<uint64_t>(B * S),
                                    static_cast<uint64_t>(ld_qkv) * 2, 64, 128);
  if (e != cudaSuccess) return e;
  if (hd == 32) return launch_attention_solo<32>(tm, p, stream);
  if (hd == 64) return launch_attention_solo<64>(tm, p, stream);
  return launch_attention_wide(tm, p, stream);
}

}  // namespace b2
