// C-ABI entry points of libb200tx.so (declared in include/b200tx.h).
//
// Conventions (the same ones the reference's ctypes cuBLASLt binding and its torch-extension
// kernels follow: transformer_benchmark/cublaslt_linear.py:63-145 maps an integer status to an
// exception; case6_exact_attention.cu:324-379 checks preconditions, launches on the caller's
// stream and checks the launch):
//   * every entry point returns int (B2_OK = 0) and takes the cudaStream_t last, as void*;
//   * pointers are device pointers the caller owns; the library allocates no device memory and
//     never synchronises the stream;
//   * on failure, b2_last_error() returns a message for the calling thread.
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "b2_common.cuh"
#include "layernorm.cuh"
#include "gemm.cuh"
#include "attention.cuh"
#include "attention_solo.cuh"
#include "attention_wide.cuh"
#include "attention_simt.cuh"
#include "peer.cuh"
#include "mask.cuh"

#define B2_API extern "C" __attribute__((visibility("default")))

namespace b2 {


static thread_local char g_last_error[512] = "";

static int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

static int check_launch(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return 0;
  return fail(3, "%s: CUDA error %d (%s)", what, static_cast<int>(e), cudaGetErrorString(e));
}

static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

cudaError_t make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                              uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return cudaErrorNotSupported;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

int device_sm_count(int device) {
  static int cache[64] = {0};
  int& c = cache[device & 63];
  if (c == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device);
    c = v > 0 ? v : 148;
  }
  return c;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static bool is_sm100(int* major_out) {
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major_out) *major_out = major * 10 + minor;
  return major == 10 && minor == 0;
}

}  // namespace b2

using namespace b2;

B2_API int b2_abi_version(void) { return 1; }

B2_API const char* b2_last_error(void) { return g_last_error; }

B2_API int b2_device_status(uint32_t* out_status, int clear) {
  if (out_status == nullptr) return fail(1, "b2_device_status: out_status is null");
  uint32_t v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_status, sizeof(v));
  if (e != cudaSuccess) return check_launch(e, "b2_device_status");
  if (clear && v != 0) {
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(zero));
    if (e != cudaSuccess) return check_launch(e, "b2_device_status(clear)");
  }
  *out_status = v;
  return 0;
}

B2_API int b2_device_status_async(uint32_t* host_dst, void* stream) {
  if (host_dst == nullptr) return fail(1, "b2_device_status_async: host_dst is null");
  return check_launch(cudaMemcpyFromSymbolAsync(host_dst, g_device_status, sizeof(uint32_t), 0,
                                                cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream)),
                      "b2_device_status_async");
}

B2_API int b2_set_wait_limit(uint64_t limit_ns) {
  const uint64_t v = limit_ns == 0 ? kWaitTimeoutNs : limit_ns;
  if (v < 1000000ull) return fail(1, "b2_set_wait_limit: limit below 1 ms");
  return check_launch(cudaMemcpyToSymbol(g_wait_limit_ns, &v, sizeof(v)), "b2_set_wait_limit");
}

B2_API int b2_test_set_fault(int fault) {
  if (fault < 0 || fault > static_cast<int>(kFaultGemmWithholdStage))
    return fail(1, "b2_test_set_fault: unknown fault %d", fault);
  const uint32_t v = static_cast<uint32_t>(fault);
  return check_launch(cudaMemcpyToSymbol(g_test_fault, &v, sizeof(v)), "b2_test_set_fault");
}

B2_API int b2_mask_lengths(const uint8_t* mask, int64_t batch, int64_t seq_len, int32_t* kv_len, uint8_t* row_mask_out,
                           uint8_t* not_prefix, void* stream) {
  if (mask == nullptr || kv_len == nullptr || not_prefix == nullptr)
    return fail(1, "b2_mask_lengths: null pointer argument");
  if (batch < 0 || seq_len <= 0) return fail(1, "b2_mask_lengths: invalid shape batch=%lld seq_len=%lld",
                                             (long long)batch, (long long)seq_len);
  if (batch > 0x7fffffffLL || seq_len > 0x7fffffffLL) return fail(2, "b2_mask_lengths: dimension exceeds 2^31");
  if (batch == 0) return 0;
  return check_launch(launch_mask_lengths(mask, batch, seq_len, kv_len, row_mask_out, not_prefix,
                                          static_cast<cudaStream_t>(stream)),
                      "b2_mask_lengths");
}

B2_API int b2_layernorm_fwd(const void* x, int x_is_bf16, const void* gamma, const void* beta, float eps, void* y,
                            float* resid_out, const uint8_t* row_mask, int64_t rows, int64_t d_model, void* stream) {
  if (x == nullptr || gamma == nullptr || beta == nullptr || y == nullptr)
    return fail(1, "b2_layernorm_fwd: null pointer argument");
  if (rows < 0 || d_model <= 0) return fail(1, "b2_layernorm_fwd: invalid shape rows=%lld d_model=%lld", (long long)rows,
                                            (long long)d_model);
  if (!(eps > 0.f)) return fail(1, "b2_layernorm_fwd: eps must be positive");
  if (rows == 0) return 0;
  if (rows > (int64_t)0x7fffffff * 8) return fail(2, "b2_layernorm_fwd: too many rows");
  return check_launch(launch_layernorm(x, x_is_bf16, static_cast<const __nv_bfloat16*>(gamma),
                                       static_cast<const __nv_bfloat16*>(beta), eps, static_cast<__nv_bfloat16*>(y),
                                       x_is_bf16 ? resid_out : nullptr, row_mask, rows, d_model,
                                       static_cast<cudaStream_t>(stream)),
                      "b2_layernorm_fwd");
}

B2_API int b2_linear_fwd(const void* a, const void* w, const void* bias, int64_t m, int64_t n, int64_t k, int epilogue,
                         void* out, int64_t ldo, const uint8_t* row_mask, int tile_n, void* stream) {
  if (a == nullptr || w == nullptr || out == nullptr) return fail(1, "b2_linear_fwd: null pointer argument");
  if (m < 0 || n <= 0 || k <= 0) return fail(1, "b2_linear_fwd: invalid shape m=%lld n=%lld k=%lld", (long long)m,
                                             (long long)n, (long long)k);
  if (epilogue < 0 || epilogue > 4)
    return fail(1, "b2_linear_fwd: unknown epilogue %d (reduce-scatter epilogues go through b2_linear_rs_fwd)",
                epilogue);
  if (n % 32 != 0) return fail(2, "b2_linear_fwd: n=%lld must be a multiple of 32", (long long)n);
  if (k % 8 != 0) return fail(2, "b2_linear_fwd: k=%lld must be a multiple of 8", (long long)k);
  if (ldo < n || ldo % 8 != 0) return fail(2, "b2_linear_fwd: ldo=%lld must be >= n and a multiple of 8", (long long)ldo);
  {
    const int bn = tile_n & 0xFFFF;
    const bool pair = (tile_n & kTilePair) != 0;
    if ((tile_n & ~(kTilePair | 0xFFFF)) != 0 || (tile_n != 0 && bn != 128 && bn != 192 && bn != 256) ||
        (pair && bn == 128))
      return fail(1, "b2_linear_fwd: tile_n must be 0, 128, 192, 256, or B2_TILE_PAIR | 192 / 256");
    if ((bn == 256 || bn == 192) && n % bn != 0)
      return fail(2, "b2_linear_fwd: an N tile of %d needs n %% %d == 0", bn, bn);
  }
  if (!aligned16(a) || !aligned16(w) || !aligned16(out) || (bias && !aligned16(bias)))
    return fail(2, "b2_linear_fwd: pointers must be 16-byte aligned");
  if (m > 0x7fffff00LL || n > 0x7fffff00LL) return fail(2, "b2_linear_fwd: dimension exceeds 2^31");
  if (m == 0) return 0;
  if (!is_sm100(nullptr)) return fail(2, "b2_linear_fwd: needs an sm_100 (B200) device");
  return check_launch(launch_gemm(static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(w),
                                  static_cast<const __nv_bfloat16*>(bias), m, n, k, epilogue, out, ldo, row_mask, tile_n,
                                  static_cast<cudaStream_t>(stream)),
                      "b2_linear_fwd");
}

B2_API int b2_linear_ln_plan(int64_t m, int64_t n, int64_t k, int sm_count, int* tile_n, int* cluster,
                             int* recommended) {
  if (m <= 0 || n <= 0 || k <= 0) return fail(1, "b2_linear_ln_plan: invalid shape");
  int sms = sm_count;
  if (sms <= 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return fail(2, "b2_linear_ln_plan: no CUDA device and no sm_count");
    sms = device_sm_count(dev);
  }
  if (m > 0x7fffff00LL || n > 0x7fffff00LL) return fail(2, "b2_linear_ln_plan: dimension exceeds 2^31");
  if (!gemm_ln_plan(m, n, k, sms, tile_n, cluster, recommended))
    return fail(2, "b2_linear_ln_plan: n=%lld has no fused plan (n %% 32 == 0 and n <= 256 or n = {128,192,256} x c, "
                "c <= 8)", (long long)n);
  return 0;
}

B2_API int b2_linear_ln_fwd(const void* a, const void* w, const void* bias, int64_t m, int64_t n, int64_t k,
                            int zero_masked_rows, float* resid, const uint8_t* row_mask, const void* gamma,
                            const void* beta, float eps, void* ln_out, void* stream) {
  if (a == nullptr || w == nullptr || resid == nullptr || gamma == nullptr || beta == nullptr || ln_out == nullptr)
    return fail(1, "b2_linear_ln_fwd: null pointer argument");
  if (m < 0 || n <= 0 || k <= 0) return fail(1, "b2_linear_ln_fwd: invalid shape m=%lld n=%lld k=%lld", (long long)m,
                                             (long long)n, (long long)k);
  if (!(eps > 0.f)) return fail(1, "b2_linear_ln_fwd: eps must be positive");
  if (k % 8 != 0) return fail(2, "b2_linear_ln_fwd: k=%lld must be a multiple of 8", (long long)k);
  if (m > 0x7fffff00LL || n > 0x7fffff00LL) return fail(2, "b2_linear_ln_fwd: dimension exceeds 2^31");
  if (!gemm_ln_plan(m > 0 ? m : 1, n, k, 0, nullptr, nullptr, nullptr))
    return fail(2, "b2_linear_ln_fwd: n=%lld has no fused plan (see b2_linear_ln_plan)", (long long)n);
  if (!aligned16(a) || !aligned16(w) || !aligned16(resid) || !aligned16(ln_out) || !aligned16(gamma) ||
      !aligned16(beta) || (bias && !aligned16(bias)))
    return fail(2, "b2_linear_ln_fwd: pointers must be 16-byte aligned");
  if (m == 0) return 0;
  if (!is_sm100(nullptr)) return fail(2, "b2_linear_ln_fwd: needs an sm_100 (B200) device");
  return check_launch(launch_gemm_ln(static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(w),
                                     static_cast<const __nv_bfloat16*>(bias), m, n, k, zero_masked_rows != 0, resid,
                                     row_mask, static_cast<const __nv_bfloat16*>(gamma),
                                     static_cast<const __nv_bfloat16*>(beta), eps, static_cast<__nv_bfloat16*>(ln_out),
                                     static_cast<cudaStream_t>(stream)),
                      "b2_linear_ln_fwd");
}

B2_API int b2_attention_rows_fwd(const void* qkv, int64_t ld_qkv, int64_t q_col, int64_t k_col, int64_t v_col,
                                 int64_t batch, int64_t seq_len, int64_t num_heads, int64_t head_dim,
                                 const int32_t* kv_len, int causal, float scale, const int64_t* q_ranges,
                                 int n_ranges, void* ctx, int64_t ld_ctx, void* stream) {
  if (qkv == nullptr || ctx == nullptr) return fail(1, "b2_attention_rows_fwd: null pointer argument");
  if (batch < 0 || seq_len < 0 || num_heads <= 0) return fail(1, "b2_attention_rows_fwd: invalid shape");
  const bool tensor_core = head_dim == 64 || head_dim == 128;
  if (!tensor_core && head_dim != 8 && head_dim != 16 && head_dim != 32 && head_dim != 256)
    return fail(2, "b2_attention_rows_fwd: head_dim=%lld not supported (8, 16, 32, 64, 128, 256)", (long long)head_dim);
  // 64 / 128: 64-column TMA boxes per head; 32 (also tensor cores, 64-column boxes starting at the
  // head's 32-column offset) and the CUDA-core head dims: 16-byte aligned column offsets.
  const int64_t col_align = tensor_core ? 64 : 8;
  if (q_col % col_align || k_col % col_align || v_col % col_align || q_col < 0 || k_col < 0 || v_col < 0)
    return fail(2, "b2_attention_rows_fwd: q/k/v column offsets must be non-negative multiples of %lld",
                (long long)col_align);
  const int64_t width = num_heads * head_dim;
  if (q_col + width > ld_qkv || k_col + width > ld_qkv || v_col + width > ld_qkv)
    return fail(1, "b2_attention_rows_fwd: q/k/v columns exceed ld_qkv");
  if (ld_qkv % 8 != 0 || ld_ctx % 8 != 0 || ld_ctx < width) return fail(2, "b2_attention_rows_fwd: bad leading dimensions");
  if (!aligned16(qkv) || !aligned16(ctx)) return fail(2, "b2_attention_rows_fwd: pointers must be 16-byte aligned");
  if (batch * seq_len > 0x7fffff00LL || batch * num_heads > 0x7fffffffLL || (seq_len + 127) / 128 > 65535)
    return fail(2, "b2_attention_rows_fwd: problem too large");
  if (!(scale > 0.f)) return fail(1, "b2_attention_rows_fwd: scale must be positive");
  if (q_ranges == nullptr || n_ranges < 1 || n_ranges > 2)
    return fail(1, "b2_attention_rows_fwd: 1 or 2 query ranges are required");
  int64_t rows = 0;
  for (int r = 0; r < n_ranges; ++r) {
    const int64_t q_begin = q_ranges[2 * r], q_count = q_ranges[2 * r + 1];
    if (q_begin < 0 || q_count <= 0 || q_begin + q_count > seq_len || q_begin % 128 != 0 ||
        (q_count % 128 != 0 && q_begin + q_count != seq_len))
      return fail(1, "b2_attention_rows_fwd: query rows [%lld, +%lld) must be non-empty, start on a multiple of 128 "
                  "and end on one or at seq_len", (long long)q_begin, (long long)q_count);
    if (r == 1 && q_begin < q_ranges[0] + q_ranges[1])
      return fail(1, "b2_attention_rows_fwd: the second query range must start after the first one ends");
    rows += q_count;
  }
  if (batch == 0 || seq_len == 0 || rows == 0) return 0;
  if (!is_sm100(nullptr)) return fail(2, "b2_attention_rows_fwd: needs an sm_100 (B200) device");
  return check_launch(launch_attention(static_cast<const __nv_bfloat16*>(qkv), ld_qkv, q_col, k_col, v_col, batch,
                                       seq_len, num_heads, head_dim, kv_len, causal, scale,
                                       static_cast<__nv_bfloat16*>(ctx), ld_ctx, static_cast<cudaStream_t>(stream), q_ranges,
                                       n_ranges),
                      "b2_attention_rows_fwd");
}

B2_API int b2_attention_fwd(const void* qkv, int64_t ld_qkv, int64_t q_col, int64_t k_col, int64_t v_col,
                            int64_t batch, int64_t seq_len, int64_t num_heads, int64_t head_dim, const int32_t* kv_len,
                            int causal, float scale, void* ctx, int64_t ld_ctx, void* stream) {
  const int64_t whole[2] = {0, seq_len};
  if (seq_len == 0 && batch >= 0 && num_heads > 0) return 0;
  const int rc = b2_attention_rows_fwd(qkv, ld_qkv, q_col, k_col, v_col, batch, seq_len, num_heads, head_dim, kv_len,
                                       causal, scale, whole, 1, ctx, ld_ctx, stream);
  if (rc != 0) {
    std::string msg = g_last_error;
    const std::string from = "b2_attention_rows_fwd";
    if (msg.compare(0, from.size(), from) == 0) msg = "b2_attention_fwd" + msg.substr(from.size());
    snprintf(g_last_error, sizeof(g_last_error), "%s", msg.c_str());
  }
  return rc;
}

B2_API int b2_add_layernorm_fwd(float* resid, const float* delta, const void* bias, const uint8_t* row_mask,
                                int flags, const void* gamma, const void* beta, float eps, void* y, int64_t rows,
                                int64_t d_model, void* stream) {
  if (resid == nullptr || delta == nullptr || gamma == nullptr || beta == nullptr || y == nullptr)
    return fail(1, "b2_add_layernorm_fwd: null pointer argument");
  if (rows < 0 || d_model <= 0) return fail(1, "b2_add_layernorm_fwd: invalid shape");
  if (!(eps > 0.f)) return fail(1, "b2_add_layernorm_fwd: eps must be positive");
  if (flags & ~3) return fail(1, "b2_add_layernorm_fwd: unknown flags %d", flags);
  if (!add_layernorm_supported(d_model))
    return fail(2, "b2_add_layernorm_fwd: d_model=%lld not supported (128 * {1,2,4,6,8,16,32})", (long long)d_model);
  if (!aligned16(resid) || !aligned16(delta) || !aligned16(y) || (bias && !aligned16(bias)) || !aligned16(gamma) ||
      !aligned16(beta))
    return fail(2, "b2_add_layernorm_fwd: pointers must be 16-byte aligned");
  if (rows == 0) return 0;
  return check_launch(launch_add_layernorm(resid, delta, static_cast<const __nv_bfloat16*>(bias), row_mask, flags & 1,
                                           (flags >> 1) & 1, static_cast<const __nv_bfloat16*>(gamma),
                                           static_cast<const __nv_bfloat16*>(beta), eps,
                                           static_cast<__nv_bfloat16*>(y), rows, d_model,
                                           static_cast<cudaStream_t>(stream)),
                      "b2_add_layernorm_fwd");
}

B2_API int b2_peer_barrier(void* const* pads, int world, int rank, int channel, void* stream) {
  if (pads == nullptr) return fail(1, "b2_peer_barrier: pads is null");
  if (world < 1 || world > kMaxPeers) return fail(2, "b2_peer_barrier: world=%d not in [1, %d]", world, kMaxPeers);
  if (rank < 0 || rank >= world) return fail(1, "b2_peer_barrier: rank %d outside world %d", rank, world);
  if (channel < 0 || channel >= kPadChannels)
    return fail(1, "b2_peer_barrier: channel %d not in [0, %d)", channel, kPadChannels);
  PeerPads p{};
  for (int r = 0; r < world; ++r) {
    if (pads[r] == nullptr || (reinterpret_cast<uintptr_t>(pads[r]) & 3u))
      return fail(1, "b2_peer_barrier: pad of rank %d is null or misaligned", r);
    p.pad[r] = static_cast<uint32_t*>(pads[r]);
  }
  if (world == 1) return 0;
  return check_launch(launch_peer_barrier(p, world, rank, channel, static_cast<cudaStream_t>(stream)),
                      "b2_peer_barrier");
}

B2_API int b2_linear_rs_fwd(const void* a, const void* w, const void* bias, int64_t m, int64_t n, int64_t k,
                            int zero_masked_rows, void* const* peer_resid, int world, int rank, int64_t rows_per_rank,
                            int64_t ldo, const uint8_t* row_mask, int tile_n, void* stream) {
  if (a == nullptr || w == nullptr || peer_resid == nullptr) return fail(1, "b2_linear_rs_fwd: null pointer argument");
  if (m < 0 || n <= 0 || k <= 0) return fail(1, "b2_linear_rs_fwd: invalid shape");
  if (world < 1 || world > kGemmMaxPeers || rank < 0 || rank >= world)
    return fail(1, "b2_linear_rs_fwd: rank %d / world %d invalid (world <= %d)", rank, world, kGemmMaxPeers);
  if (rows_per_rank <= 0 || rows_per_rank * world < m) return fail(1, "b2_linear_rs_fwd: rows_per_rank too small");
  if (n % 32 != 0 || k % 8 != 0 || ldo < n || ldo % 8 != 0)
    return fail(2, "b2_linear_rs_fwd: n %% 32, k %% 8, ldo >= n and ldo %% 8 are required");
  if ((tile_n & ~(kTilePair | 0xFFFF)) != 0) return fail(1, "b2_linear_rs_fwd: bad tile_n");
  void* peers[kGemmMaxPeers] = {};
  for (int r = 0; r < world; ++r) {
    if (peer_resid[r] == nullptr || !aligned16(peer_resid[r]))
      return fail(2, "b2_linear_rs_fwd: residual of rank %d is null or not 16-byte aligned", r);
    peers[r] = peer_resid[r];
  }
  if (!aligned16(a) || !aligned16(w) || (bias && !aligned16(bias)))
    return fail(2, "b2_linear_rs_fwd: pointers must be 16-byte aligned");
  if (m == 0) return 0;
  if (!is_sm100(nullptr)) return fail(2, "b2_linear_rs_fwd: needs an sm_100 (B200) device");
  return check_launch(launch_gemm(static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(w),
                                  static_cast<const __nv_bfloat16*>(bias), m, n, k,
                                  zero_masked_rows ? kEpiRsResidualZero : kEpiRsResidual, peers[rank], ldo, row_mask,
                                  tile_n, static_cast<cudaStream_t>(stream), peers, world, rank, rows_per_rank),
                      "b2_linear_rs_fwd");
}

B2_API int b2_layernorm_gather_fwd(const float* x, const void* gamma, const void* beta, float eps,
                                   void* const* y_ranks, int world, const uint8_t* row_mask, int64_t rows,
                                   int64_t d_model, void* stream) {
  if (x == nullptr || gamma == nullptr || beta == nullptr || y_ranks == nullptr)
    return fail(1, "b2_layernorm_gather_fwd: null pointer argument");
  if (rows < 0 || d_model <= 0 || !(eps > 0.f)) return fail(1, "b2_layernorm_gather_fwd: invalid arguments");
  if (world < 1 || world > kGatherMaxRanks) return fail(1, "b2_layernorm_gather_fwd: world %d not in [1, 8]", world);
  if (!layernorm_gather_supported(d_model))
    return fail(2, "b2_layernorm_gather_fwd: d_model=%lld not supported (256 * {1,2,3,4,8,16})", (long long)d_model);
  GatherDst dst{};
  for (int r = 0; r < world; ++r) {
    if (y_ranks[r] == nullptr || !aligned16(y_ranks[r]))
      return fail(2, "b2_layernorm_gather_fwd: destination of rank %d is null or not 16-byte aligned", r);
    dst.rank_rows[r] = static_cast<__nv_bfloat16*>(y_ranks[r]);
  }
  if (!aligned16(x) || !aligned16(gamma) || !aligned16(beta))
    return fail(2, "b2_layernorm_gather_fwd: pointers must be 16-byte aligned");
  if (rows == 0) return 0;
  return check_launch(launch_layernorm_gather(x, static_cast<const __nv_bfloat16*>(gamma),
                                              static_cast<const __nv_bfloat16*>(beta), eps, dst, world, row_mask, rows,
                                              d_model, static_cast<cudaStream_t>(stream)),
                      "b2_layernorm_gather_fwd");
}

B2_API int b2_linear_bcast_fwd(const void* a, const void* w, const void* bias, int64_t m, int64_t n, int64_t k,
                               void* const* peer_out, int world, int rank, int64_t col_begin, int64_t ldo, int tile_n,
                               void* stream) {
  if (a == nullptr || w == nullptr || peer_out == nullptr) return fail(1, "b2_linear_bcast_fwd: null pointer argument");
  if (m < 0 || n <= 0 || k <= 0) return fail(1, "b2_linear_bcast_fwd: invalid shape");
  if (world < 1 || world > kGemmMaxPeers || rank < 0 || rank >= world)
    return fail(1, "b2_linear_bcast_fwd: rank %d / world %d invalid (world <= %d)", rank, world, kGemmMaxPeers);
  if (n % 32 != 0 || k % 8 != 0 || ldo < n || ldo % 8 != 0)
    return fail(2, "b2_linear_bcast_fwd: n %% 32, k %% 8, ldo >= n and ldo %% 8 are required");
  if (col_begin < 0 || col_begin > n || col_begin % 32 != 0)
    return fail(1, "b2_linear_bcast_fwd: col_begin must be a multiple of 32 in [0, n]");
  if ((tile_n & ~(kTilePair | 0xFFFF)) != 0) return fail(1, "b2_linear_bcast_fwd: bad tile_n");
  void* peers[kGemmMaxPeers] = {};
  for (int r = 0; r < world; ++r) {
    if (peer_out[r] == nullptr || !aligned16(peer_out[r]))
      return fail(2, "b2_linear_bcast_fwd: output of rank %d is null or not 16-byte aligned", r);
    peers[r] = peer_out[r];
  }
  if (!aligned16(a) || !aligned16(w) || (bias && !aligned16(bias)))
    return fail(2, "b2_linear_bcast_fwd: pointers must be 16-byte aligned");
  if (m == 0) return 0;
  if (!is_sm100(nullptr)) return fail(2, "b2_linear_bcast_fwd: needs an sm_100 (B200) device");
  return check_launch(launch_gemm(static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(w),
                                  static_cast<const __nv_bfloat16*>(bias), m, n, k, kEpiBiasPeers, peers[rank], ldo,
                                  nullptr, tile_n, static_cast<cudaStream_t>(stream), peers, world, rank, 0, col_begin),
                      "b2_linear_bcast_fwd");
}
