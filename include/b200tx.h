/*
 * b200tx.h — C-ABI of libb200tx.so, the sm_100a (B200) kernels behind the forward pass of the
 * TikTok TechJam 2026 Track 3 Transformer encoder stack (Sober7135/TikTokTechJam2026Track3).
 *
 * The reference computes this forward pass with ATen calls inside
 * BaselineTransformer.forward (transformer_benchmark/models.py:909-919) and reaches native code
 * through two FFI styles: ctypes over a C library (transformer_benchmark/cublaslt_linear.py:63-145)
 * and torch extensions taking tensors (e.g. case6_exact_layer_norm.py:98-121). This header is the
 * ctypes-style boundary for the whole path: plain pointers, int64 sizes, int status, the CUDA
 * stream last as void*. No torch types appear here.
 *
 * Conventions for every entry point:
 *   - returns B2_OK (0) on success; B2_E_INVALID (1) for a bad argument, B2_E_UNSUPPORTED (2) for
 *     a shape/alignment/device the kernels do not cover, B2_E_CUDA (3) for a CUDA error at launch;
 *     b2_last_error() then describes the failure (per calling thread);
 *   - pointers are device pointers owned by the caller; the library allocates no device memory,
 *     keeps no pointer after the call returns (work is enqueued on `stream`) and never
 *     synchronises the stream;
 *   - bf16 means IEEE bfloat16 stored as uint16; row-major throughout;
 *   - device-side pipeline timeouts (a stuck mbarrier wait) do not trap: they set a status word
 *     read with b2_device_status().
 */
#ifndef B200TX_H_
#define B200TX_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B2_OK 0
#define B2_E_INVALID 1
#define B2_E_UNSUPPORTED 2
#define B2_E_CUDA 3

/* Epilogues of b2_linear_fwd (acc = A W^T in fp32). */
#define B2_EPI_BIAS 0           /* out bf16 = bf16(acc + bias)                          */
#define B2_EPI_BIAS_GELU 1      /* out bf16 = bf16(gelu_erf(bf16(acc + bias)))           */
#define B2_EPI_RESIDUAL 2       /* out f32 (in place) = mask ? out + acc + bias : out    */
#define B2_EPI_RESIDUAL_ZERO 3  /* out f32 (in place) = mask ? out + acc + bias : 0      */
#define B2_EPI_STORE_F32 4      /* out f32 = acc (+ bias if non-null)                     */

/* b2_linear_fwd tile_n flag: the 2-SM variant (a CTA pair computes 256-row tiles with
 * tcgen05.mma.cta_group::2), combined with an N tile of 192 or 256. */
#define B2_TILE_PAIR 0x10000

/* ABI revision of this header (1). */
int b2_abi_version(void);

/* Message describing the last failed call on this thread ("" if none). */
const char* b2_last_error(void);

/* Reads (and with clear != 0 resets) the current device's pipeline status word:
 * 0 = no kernel gave up waiting since the last clear; otherwise (kernel << 16) | (site << 8) |
 * reason, kernel 2 = linear, 3 = attention. Synchronous: it waits for the device. */
int b2_device_status(uint32_t* out_status, int clear);

/* Enqueues a copy of the current device's status word (the value b2_device_status reads, not
 * cleared) into host_dst on `stream`, behind the work already enqueued there; host_dst should be
 * pinned host memory, valid until the copy completes. Lets a caller check every forward pass for
 * a pipeline timeout without synchronising: read *host_dst once an event recorded after this call
 * has completed. No counterpart in the reference (its kernels have no bounded waits). */
int b2_device_status_async(uint32_t* host_dst, void* stream);

/* Sets the current device's limit for one pipeline wait (mbarrier, peer flag) in nanoseconds;
 * 0 restores the default of 4 s, values below 1 ms are rejected. Applies to kernels launched after
 * the call (synchronous copy to the device). No counterpart in the reference. */
int b2_set_wait_limit(uint64_t limit_ns);

/* Test-only fault selector of the current device, for checking the bounded waits without
 * faulting the GPU: 0 = none (default); 1 = in the next b2_linear_fwd launches with one-CTA tiles,
 * CTA 0's producer neither arms nor loads its first pipeline stage, so the MMA issuer's wait for
 * it runs out after the wait limit: the kernel records status (2 << 16) | (3 << 8) | 1, leaves its
 * loops, frees its tensor memory and returns; that CTA's output tile is not written. Reset to 0
 * after use. No counterpart in the reference. */
int b2_test_set_fault(int fault);

/*
 * The valid-token mask of a forward pass turned into what the kernels take, in one launch: the
 * reference's padding masks are prefixes (generate_random_case, transformer_benchmark/cases.py:87-97),
 * consumed as per-sequence key lengths by the attention (models.py:63-66) and as a row mask by the
 * padded-row zeroing (models.py:78-79, 736-737, 917-918).
 *   mask        [batch, seq_len] bool as bytes (0 / nonzero)
 *   kv_len      [batch] int32 out: the number of nonzero entries of row b
 *   row_mask_out [batch * seq_len] uint8 out (0 / 1), or NULL when the caller passes the mask
 *               itself as the row mask
 *   not_prefix  [batch] uint8 out: 1 where row b is not a prefix of length kv_len[b], else 0
 */
int b2_mask_lengths(const uint8_t* mask, int64_t batch, int64_t seq_len, int32_t* kv_len, uint8_t* row_mask_out,
                    uint8_t* not_prefix, void* stream);

/*
 * LayerNorm over the last dimension: y = (x - mean) / sqrt(var + eps) * gamma + beta, fp32
 * statistics, bf16 y. Replaces nn.LayerNorm in BaselineTransformerBlock (models.py:721, 723) and
 * final_norm (models.py:907) with the padded-row zeroing of models.py:917-918 fused in:
 * rows with row_mask[r] == 0 get y = 0 (row_mask may be NULL).
 *   x          [rows, d_model] fp32 (x_is_bf16 = 0) or bf16 (x_is_bf16 = 1)
 *   gamma,beta [d_model] bf16
 *   y          [rows, d_model] bf16
 *   resid_out  NULL, or (x_is_bf16 = 1 only) [rows, d_model] fp32 receiving float(x)
 */
int b2_layernorm_fwd(const void* x, int x_is_bf16, const void* gamma, const void* beta, float eps, void* y,
                     float* resid_out, const uint8_t* row_mask, int64_t rows, int64_t d_model, void* stream);

/*
 * Residual update fused with the LayerNorm that follows it, for tensor-parallel blocks whose
 * out_proj / ffn_out partial sums are all-reduced before the residual add (the reference adds
 * them in BaselineTransformerBlock.forward, models.py:733-737):
 *   resid = row_mask[r] ? resid + delta + bias : (flags & 1 ? 0 : resid)    (in place, fp32)
 *   y     = LayerNorm(resid) in bf16; with flags & 2, rows with row_mask[r] == 0 get y = 0
 *   delta [rows, d_model] fp32 (the all-reduced partial); bias [d_model] bf16 or NULL;
 *   row_mask [rows] uint8 or NULL (all rows kept). d_model = 128 * {1, 2, 4, 6, 8, 16, 32}.
 */
int b2_add_layernorm_fwd(float* resid, const float* delta, const void* bias, const uint8_t* row_mask, int flags,
                         const void* gamma, const void* beta, float eps, void* y, int64_t rows, int64_t d_model,
                         void* stream);

/*
 * out = epilogue(A W^T + bias) on tcgen05 tensor cores (fp32 accumulate in TMEM, TMA-fed).
 * Replaces the nn.Linear calls of a block — packed q/k/v_proj (models.py:51-53), out_proj (:76),
 * ffn_in and ffn_out (:734) — with the pointwise work after them fused (see B2_EPI_*).
 *   a    [m, k] bf16;  w [n, k] bf16 (nn.Linear weight layout);  bias [n] bf16 or NULL
 *   out  [m, ldo] bf16 (B2_EPI_BIAS, B2_EPI_BIAS_GELU) or fp32 (others)
 *   row_mask [m] uint8 or NULL (residual epilogues only)
 *   tile_n 0 = choose; 128 / 192 / 256 = one CTA per 128 x tile_n tile; B2_TILE_PAIR | 192 / 256 =
 *          a CTA pair per 256 x tile_n tile (192 and 256 need n to be a multiple)
 * Requires n % 32 == 0, k % 8 == 0, ldo % 8 == 0, 16-byte aligned pointers, an sm_100 device.
 */
int b2_linear_fwd(const void* a, const void* w, const void* bias, int64_t m, int64_t n, int64_t k, int epilogue,
                  void* out, int64_t ldo, const uint8_t* row_mask, int tile_n, void* stream);

/*
 * A residual GEMM and the LayerNorm after it in one launch: resid = mask ? resid + A W^T + bias :
 * (zero_masked_rows ? 0 : resid), then ln_out = LayerNorm(resid) with gamma, beta, eps (biased
 * variance, fp32 statistics, bf16 out; every row normalised, masked ones included, as nn.LayerNorm
 * does). Replaces out_proj + residual add + norm2 (models.py:76-79, 733, 723) and ffn_out +
 * residual add + masked_fill + the next block's norm1 (:734-737, 721). A cluster of n / tile_n
 * CTAs computes each 128-row stripe, and the CTAs exchange row sums through distributed shared
 * memory, so the residual is read and written once and the LayerNorm needs no launch of its own.
 *   a [m, k] bf16; w [n, k] bf16; bias [n] bf16 or NULL; resid [m, n] fp32 (in place);
 *   row_mask [m] uint8 or NULL; gamma, beta [n] bf16; ln_out [m, n] bf16
 * Requires n % 32 == 0 and a plan (b2_linear_ln_plan) for n: n <= 256, or n = tile_n x c with
 * tile_n in {128, 192, 256} and c <= 8; k % 8 == 0; 16-byte aligned pointers; an sm_100 device.
 */
int b2_linear_ln_fwd(const void* a, const void* w, const void* bias, int64_t m, int64_t n, int64_t k,
                     int zero_masked_rows, float* resid, const uint8_t* row_mask, const void* gamma, const void* beta,
                     float eps, void* ln_out, void* stream);

/*
 * The tile b2_linear_ln_fwd uses for n output columns (no device work): returns 0 and sets *tile_n
 * and *cluster (CTAs per 128-row stripe; n <= 256: one CTA, else a power-of-two cluster first,
 * then the widest tile), and *recommended = 1 where the fused launch is expected to beat
 * b2_linear_fwd + b2_layernorm_fwd (0 for every n in this build: measured slower on B200 at the
 * benchmark sizes). The plan depends on n only, so a row's output never depends on m (batch shards
 * reproduce the full batch bit for bit). Returns 2 when n has no plan. m and k are
 * validated only; sm_count is unused (kept for the signature).
 */
int b2_linear_ln_plan(int64_t m, int64_t n, int64_t k, int sm_count, int* tile_n, int* cluster, int* recommended);

/*
 * Multi-head self-attention core (BaselineSelfAttention.forward, models.py:55-75) as one
 * flash-style tcgen05 kernel: scores = q k^T * scale, causal (key > query) and/or padding
 * (key >= kv_len[b]) masked to -inf, fp32 softmax, context = p v written as bf16 to
 * ctx[(b*seq_len + s) * ld_ctx + h*head_dim + d]. Query rows at or past kv_len[b] in whole
 * 128-row tiles are not written.
 *   qkv     [batch*seq_len, ld_qkv] bf16; head h of Q/K/V at columns q_col/k_col/v_col + h*head_dim
 *   kv_len  [batch] int32 (valid-key prefix length per sequence) or NULL (= seq_len)
 * Requires head_dim in {64, 128} (tcgen05 tensor cores; q/k/v_col multiples of 64), 32 (tensor
 * cores; q/k/v_col multiples of 8) or {8, 16, 256} (CUDA cores; q/k/v_col multiples of 8),
 * ld_qkv % 8 == 0, an sm_100 device.
 */
int b2_attention_fwd(const void* qkv, int64_t ld_qkv, int64_t q_col, int64_t k_col, int64_t v_col, int64_t batch,
                     int64_t seq_len, int64_t num_heads, int64_t head_dim, const int32_t* kv_len, int causal,
                     float scale, void* ctx, int64_t ld_ctx, void* stream);

/*
 * b2_attention_fwd for some query rows of every sequence only: q_ranges holds n_ranges (1 or 2)
 * pairs (q_begin, q_count); keys are all of the sequence's valid keys and the causal mask uses
 * absolute positions. Used by context parallelism, where a rank owns two query chunks of a long
 * sequence and holds every key (one launch for both; the later range's work is issued first).
 * Each q_begin is a multiple of 128 and each q_count too, unless its range ends at seq_len; the
 * second range starts after the first ends. Other context rows are not written.
 */
int b2_attention_rows_fwd(const void* qkv, int64_t ld_qkv, int64_t q_col, int64_t k_col, int64_t v_col,
                          int64_t batch, int64_t seq_len, int64_t num_heads, int64_t head_dim, const int32_t* kv_len,
                          int causal, float scale, const int64_t* q_ranges, int n_ranges, void* ctx, int64_t ld_ctx,
                          void* stream);

/*
 * Tensor-parallel reduce-scatter fused into a residual GEMM: out = A W^T (+ bias) is added with
 * fp32 atomics (system scope) into the residual copy of the rank that owns each row — rank
 * r / rows_per_rank — so after every rank's call each owner holds its rows' full sum. No
 * counterpart in the reference (one GPU); replaces out_proj / ffn_out + NCCL all-reduce
 * (models.py:76, 734) under head / FFN-column tensor parallelism.
 *   peer_resid  host array of `world` device pointers: every rank's fp32 residual [m, ldo] as
 *               mapped into this process (peer memory over NVLink); the caller's is peer_resid[rank]
 *   bias        [n] bf16, passed on one rank only
 *   zero_masked_rows  rows with row_mask 0 are set to 0 by their owner (ffn_out), else kept
 * The caller orders the owners' reads of the residual against the adds (b2_peer_barrier).
 */
int b2_linear_rs_fwd(const void* a, const void* w, const void* bias, int64_t m, int64_t n, int64_t k,
                     int zero_masked_rows, void* const* peer_resid, int world, int rank, int64_t rows_per_rank,
                     int64_t ldo, const uint8_t* row_mask, int tile_n, void* stream);

/*
 * b2_linear_fwd with epilogue B2_EPI_BIAS whose output columns [col_begin, n) are also stored into
 * every other context-parallel rank's copy of the output (NVLink peer stores from the epilogue):
 * the packed Q/K/V projection of a rank's token rows with K and V all-gathered on the fly. No
 * counterpart in the reference (one GPU); replaces q/k/v_proj (models.py:51-53) plus the K/V
 * exchange of context parallelism.
 *   peer_out  host array of `world` device pointers: every rank's output [m, ldo] bf16 as mapped
 *             into this process; the caller's is peer_out[rank]
 * The caller orders the peers' reads of their outputs against these stores (b2_peer_barrier).
 */
int b2_linear_bcast_fwd(const void* a, const void* w, const void* bias, int64_t m, int64_t n, int64_t k,
                        void* const* peer_out, int world, int rank, int64_t col_begin, int64_t ldo, int tile_n,
                        void* stream);

/*
 * LayerNorm of fp32 rows (x [rows, d_model]) written as bf16 into the same rows of every
 * tensor-parallel rank's buffer: the all-gather of a LayerNorm whose rows are split over the ranks
 * (nn.LayerNorm, models.py:721, 723, 907; no counterpart for the gather). y_ranks is a host array
 * of `world` device pointers (each rank's destination for the first row, as mapped into this
 * process — the caller's own buffer and NVLink peer buffers). row_mask 0 rows are written as 0.
 * d_model = 256 * {1, 2, 3, 4, 8, 16}. The caller orders the readers with b2_peer_barrier.
 */
int b2_layernorm_gather_fwd(const float* x, const void* gamma, const void* beta, float eps, void* const* y_ranks,
                            int world, const uint8_t* row_mask, int64_t rows, int64_t d_model, void* stream);

/*
 * Cross-GPU barrier for tensor-parallel runs whose all-reduce is fused into the GEMM epilogues
 * (b2_linear_rs_fwd) and the all-gather into the LayerNorm (b2_layernorm_gather_fwd). No
 * counterpart in the reference, which runs on one GPU; in this build
 * it takes the place of the synchronisation an NCCL all-reduce gives.
 *   pads    host array of `world` device pointers: every rank's flag pad (4 x 8 uint32, zeroed
 *           before first use) as mapped into this process (e.g. symmetric memory buffer_ptrs)
 *   channel 0..3; ranks must use channels in the same order
 * Enqueues one block on `stream` that signals every peer and waits for every peer's signal
 * (release/acquire at system scope). A wait that exceeds 4 s records a status for
 * b2_device_status() instead of hanging. world == 1 is a no-op.
 */
int b2_peer_barrier(void* const* pads, int world, int rank, int channel, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200TX_H_ */
