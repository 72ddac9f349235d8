/*
 * lbw.h -- C ABI of the B200 (sm_100a) causal-fast DiT block forward.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t passed as void*,
 * enqueues its kernels on that stream and returns an int status (LBW_OK = 0). On failure the
 * message is available from lbw_last_error(). Nothing here allocates per call except the
 * one 64-byte device status word per device created on first use; all scratch buffers are the
 * caller's. Tensors are row-major and contiguous unless a row stride ("ld") is given; bf16 means
 * IEEE bfloat16 stored as uint16.
 *
 * Reference interfaces (yahavb/lingbot-world-v2) each entry point replaces are cited beside it.
 */
#ifndef LBW_H_
#define LBW_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LBW_VERSION 1

enum lbw_status {
  LBW_OK = 0,
  LBW_ERR_INVALID = 1,     /* null pointer, inconsistent arguments          */
  LBW_ERR_SHAPE = 2,       /* shape outside what the kernels tile            */
  LBW_ERR_ALIGN = 3,       /* pointer or row stride not 16-byte aligned      */
  LBW_ERR_CUDA = 4,        /* CUDA runtime/driver error                      */
  LBW_ERR_TIMEOUT = 5,     /* a kernel's bounded wait ran out                */
  LBW_ERR_UNSUPPORTED = 6  /* configuration this build does not implement   */
};

/* ---- library plumbing --------------------------------------------------------------- */
int lbw_version(void);
/* Copies this thread's last error message into buf (always NUL-terminated). */
int lbw_last_error(char* buf, size_t n);
const char* lbw_status_string(int code);
/* Synchronises `stream`, reads and clears the device status words of the current device (the library's, and
 * the one of lbw_linear_rmsnorm_noalloc); allocates nothing. Returns LBW_ERR_TIMEOUT (device_code =
 * 0x100 | site) if a kernel wait ran out. */
int lbw_check_device_status(void* stream, int* device_code);
/* Per-device setup, optional (the per-device handle the port plans as lbw_init(device, nccl_comm); the
 * sequence-parallel exchange here runs over CUDA IPC, so no communicator is passed). Creates on `device`, now
 * instead of on first use, what the library keeps per device: the device status word (a 64-byte allocation)
 * and the peer pull streams and events, so that a caller which later hands the rest of device memory to a
 * pool of its own has the library's allocations made first. Idempotent; the caller's current context is
 * current again on return. LBW_ERR_INVALID for a device that does not exist.
 * Replaces: nothing in the reference (its NKI kernels keep no per-device state); planned boundary item. */
int lbw_init(int device);
/* Waits for `device` (cudaDeviceSynchronize: no exchange may still be waiting on a peer), then frees the
 * status word and destroys the pull streams and events. The next call that needs them creates them again.
 * Peer buffers and registered flag blocks belong to the caller (lbw_peer_buffer_close,
 * lbw_host_flags_unregister). */
int lbw_destroy(int device);

/* ---- chunk attention ----------------------------------------------------------------
 * out[q, h*128:(h+1)*128] = softmax(scale * Q_h K_hᵀ + bias) V_h over the concatenation of
 * n_chunks KV chunks (chunk i has chunk_rows[i] keys), exact (online-softmax) in fp32.
 * q/out: [q_rows, heads*128] bf16 with row strides ldq/ldo; each chunk: [rows, heads*128] bf16
 * with row stride ldkv (the [1, L, n, d] cache layout). key_bias: optional fp32 per key of the
 * concatenation, in natural-log units (the cross_dedup log-multiplicity), or NULL.
 * Replaces: wan/modules/attention.py:1048-1058 exact_attention_chunks (SDPA over torch.cat of
 * the chunks, :1134-1143), attention.py:248-265 const_max_ag_attention (attention part; the
 * all-gather is done by the caller over NCCL), attention.py:532-554 cross_attention_dedup and
 * the cross-attention call attention(q, k, v, is_cross_attn=True) in model_fast.py:2830. */
int lbw_chunk_attention(const void* q, long long ldq, int q_rows, int heads, const void* const* k_chunks,
                        const void* const* v_chunks, const int* chunk_rows, int n_chunks, long long ldkv,
                        const float* key_bias, float softmax_scale, void* out, long long ldo, void* stream);

/* Split-KV form of lbw_chunk_attention: the window's 128-key tiles are divided into n_splits contiguous
 * ranges (1 <= n_splits <= number of tiles), one CTA per (query block, head, range). Each range writes its
 * unnormalised fp32 output to part_o[slot][q_rows][heads][128] and (running max m in log2 units, row sum l)
 * to part_ml[slot][q_rows][heads][2], slot = slot0 + range. Used to fill the GPU when a rank has few query
 * rows and to attend the cached chunks while the new chunk's K/V are still being all-gathered (the
 * reference's merged per-chunk partials, wan/modules/attention.py:963-1045, cte_partial / cte_merge). */
int lbw_chunk_attention_partial(const void* q, long long ldq, int q_rows, int heads, const void* const* k_chunks,
                                const void* const* v_chunks, const int* chunk_rows, int n_chunks, long long ldkv,
                                const float* key_bias, float softmax_scale, int n_splits, float* part_o,
                                float* part_ml, int slot0, void* stream);
/* lbw_chunk_attention (out != NULL, n_splits = 1) or lbw_chunk_attention_partial (part_o/part_ml) where the
 * chunks gate_chunk..n_chunks-1 may still be arriving: each CTA waits (bounded) until *gate_flag reaches
 * gate_value (wrap-safe) before its first load from them. gate_flag is written by a stream memory operation
 * on another stream once copy engines have filled those chunks (lbw_sp_kv_gather writes it), so the gather of
 * the new chunk's K/V runs under the attention of the cached chunks without a separate launch for the new
 * chunk (the reference overlaps the same way, wan/modules/model_fast.py:2033-2110). No key bias.
 * The wait's limit is LBW_GATE_TIMEOUT_S seconds of the GPU's global timer (environment, read per call; default
 * 120, above the exchange watchdog's default 60 s, whose release of a lost peer's flags opens the gate first);
 * when it runs out the kernel returns and lbw_check_device_status reports device code 0x123. */
int lbw_chunk_attention_gated(const void* q, long long ldq, int q_rows, int heads, const void* const* k_chunks,
                              const void* const* v_chunks, const int* chunk_rows, int n_chunks, long long ldkv,
                              float softmax_scale, void* out, long long ldo, int n_splits, float* part_o,
                              float* part_ml, int slot0, const unsigned int* gate_flag, unsigned int gate_value,
                              int gate_chunk, void* stream);
/* out[q, h*128:] = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s over slots 0..n_slots-1 (M = max m_s), bf16.
 * Replaces attention.py:963-990 cte_merge. */
int lbw_attention_merge(const float* part_o, const float* part_ml, int n_slots, int q_rows, int heads, void* out,
                        long long ldo, void* stream);
/* lbw_chunk_attention balanced over the SMs of the current device: a window is one head's pair of 128-row query
 * tiles against every key (ceil(q_rows / 256) * heads of them); whole windows run in full waves, and the windows
 * past the last full wave are cut into `pieces` key ranges (0: chosen here) that fill the SMs the last wave
 * leaves idle, followed by a merge of those windows only (two launches on `stream`). part_o / part_ml hold
 * ws_blocks blocks of [256][128] / [256][2] fp32; lbw_attention_tail_plan gives the n_tail * pieces needed
 * (0 when nothing is cut: the workspace may then be NULL). gate_flag / gate_value / gate_chunk as in
 * lbw_chunk_attention_gated (gate_chunk = n_chunks: no gate; a gated launch takes no key bias). Replaces the
 * same call as lbw_chunk_attention (wan/modules/attention.py:1048-1058) and, gated, the per-chunk partials
 * merged after the all-gather (attention.py:963-1045). */
int lbw_attention_tail_plan(int q_rows, int heads, const int* chunk_rows, int n_chunks, int pieces, int* n_tail,
                            int* pieces_used);
int lbw_chunk_attention_tail(const void* q, long long ldq, int q_rows, int heads, const void* const* k_chunks,
                             const void* const* v_chunks, const int* chunk_rows, int n_chunks, long long ldkv,
                             const float* key_bias, float softmax_scale, void* out, long long ldo, int pieces,
                             float* part_o, float* part_ml, long long ws_blocks, const unsigned int* gate_flag,
                             unsigned int gate_value, int gate_chunk, void* stream);

/* ---- tensor-core linear layers (bf16 x bf16 -> fp32 accumulate) ------------------------
 * All weights are nn.Linear layout [n_out, k_in] bf16; K must be a multiple of 64, N of 32. */

/* out[m, n] = bf16(a[m,:] · w[n,:] + bias[n]). Replaces torch nn.Linear in bf16
 * (e.g. model_fast.py:2870-2872 ffn[0], cross k/v projections :2789-2790). */
int lbw_gemm_bf16(const void* a, long long lda, const void* w, long long ldw, const void* bias, void* out,
                  long long ldo, int m, int n, int k, void* stream);

/* Fused q|k|v projection of h [m, c] with w_qkv = [Wq; Wk; Wv] [3c, c], b_qkv [3c]:
 * q_raw, k_raw [m, c] bf16 and their row sums of squares ss_q, ss_k [m] fp32 (zeroed here),
 * v written to v_out rows v_row_off.. with row stride ldv (the KV-cache destination chunk).
 * Replaces: qkv_fn's projections, model_fast.py:1821-1828 (q/k/v Linears), and the V half of
 * the cache write :2398-2409 / qk_post.qk_ss (kernels/qk_post.py:404-413). */
int lbw_qkv_proj(const void* h, const void* w_qkv, const void* b_qkv, int m, int c, void* q_raw, void* k_raw,
                 float* ss_q, float* ss_k, void* v_out, long long ldv, int v_row_off, void* stream);

/* out = bf16(a w^T + bias) [m, n] plus its row sums of squares ss [m] (zeroed here).
 * Replaces: WanCrossAttention q projection before norm_q, model_fast.py:2774-2777. */
int lbw_linear_rowss(const void* a, const void* w, const void* bias, int m, int n, int k, void* out, float* ss,
                     void* stream);

/* x[m, n] (fp32, in place) += bf16(a w^T + bias) * gate[n]; then, if film_scale is given,
 * x = bf16(1 + film_scale) * x + film_shift (film tensors [m, n] bf16). gate may be NULL (= 1).
 * Replaces: _out_proj + the gated residual and camera FiLM, model_fast.py:2709-2750, :3063-3089;
 * the cross-attention residual :3098-3100; the FFN residual x + y * e5, :3110-3111. */
int lbw_linear_residual(const void* a, const void* w, const void* bias, int m, int n, int k, float* x,
                        const float* gate, const void* film_scale, const void* film_shift, void* stream);

/* out[m, n] = bf16(GELU_tanh(bf16(a w^T) + bias)); with mx_qdq != 0 each 32-column block is then
 * MXFP8 quantise-dequantised: the FFN-up matmul with the kernels/ffn_epi.py:15-37 bias+GELU
 * epilogue and the activation quantisation of the down projection (kernels/ffn_mx.py:159-182),
 * computed on the bf16 tensor pipe. Replaces ffn[0] + ffn[1] (model_fast.py:2870-2872). */
int lbw_linear_gelu(const void* a, const void* w, const void* bias, int m, int n, int k, void* out, int mx_qdq,
                    void* stream);

/* Allocation-free linear + RMSNorm: out[m, n] = bf16(bf16(y * rsqrt(mean_n(y^2) + eps)) * gamma) with
 * y = bf16(a w^T + bias) -- the result of lbw_linear_rowss followed by lbw_rmsnorm_rope without RoPE, but
 * the per-row sums of squares are kept in a fixed 256 KB array inside the library (m <= 65536 rows;
 * larger m returns LBW_ERR_SHAPE) instead of a caller buffer, and no device memory is ever allocated
 * (its bounded-wait timeouts go to a second fixed word in the library, which lbw_check_device_status
 * reads and clears without allocating; after a timeout the RMSNorm pass leaves out unchanged). It exists
 * for callers that cannot allocate: runtimes that reserve all device memory for their own pool up front
 * and plugins hosted by another framework with no allocator to offer. Every GPU that loads the library
 * holds the array until the process exits. The first call in each device context looks up the arrays'
 * device addresses (make that first call before any stream capture). All calls share the one array, so
 * calls that overlap on the GPU (other streams, other threads) race; serialise them. No counterpart in
 * the reference: it is an addition of this library. */
int lbw_linear_rmsnorm_noalloc(const void* a, const void* w, const void* bias, const void* gamma, int m, int n, int k,
                               float eps, void* out, void* stream);

/* out[m, n] = bf16(act(bf16(a w^T + bias))) (+ addend[m, n], rounded to bf16); act = SiLU if silu != 0.
 * The block's camera-FiLM MLP: cam_injector_layer1 + SiLU and cam_injector_layer2 + the camera
 * embedding (CausalWanAttentionBlock.cam_film, model_fast.py:2882-2891). */
int lbw_linear_act(const void* a, const void* w, const void* bias, const void* addend, int silu, int m, int n, int k,
                   void* out, void* stream);

/* ---- row kernels ----------------------------------------------------------------------- */

/* h[m, c] = LN(x)[m, :] * (1 + scale) + shift (fp32 math, eps, no affine) -> bf16, or with
 * affine weight/bias instead (scale/shift NULL). If mx_qdq != 0 every 32-column block of the
 * output is MXFP8 quantise-dequantised. Replaces: WanLayerNorm + adaLN modulation
 * (model_fast.py:3045, :3101; model.py:145-156), norm3 (:2865-2867), glue.ln_mod
 * (kernels/glue.py:69-166). */
int lbw_layernorm_mod(const float* x, int m, int c, float eps, const float* scale, const float* shift,
                      const float* weight, const float* bias, int mx_qdq, void* out, void* stream);

/* As lbw_layernorm_mod with scale/shift, but the output is MXFP8: E4M3 codes data[m, c] and E8M0 scales in
 * the tiled layout of lbw_mx_quantize (rows padded to 128; c % 128 == 0). This is the FFN input
 * h = (LN(x)(1 + e4) + e3).to(bf16) (model_fast.py:3101) quantised for the MXFP8 FFN (kernels/ffn_mx.py:159-182). */
int lbw_layernorm_mod_mx(const float* x, int m, int c, float eps, const float* scale, const float* shift, void* data,
                         void* scales, void* stream);
/* lbw_layernorm_mod_mx with the codes in element format fmt: LBW_MX_E4M3 or LBW_MX_E5M2 (the reference's
 * LINGBOT_MX_FP8=float8_e5m2, kernels/ffn_mx.py:8,18). */
int lbw_layernorm_mod_mx_fmt(const float* x, int m, int c, float eps, const float* scale, const float* shift, int fmt,
                             void* data, void* scales, void* stream);
/* As lbw_layernorm_mod_mx with the affine weight/bias of norm3 (fp32 [c]) instead of the modulation: the
 * cross-attention q input LN(x) * w3 + b3 (model_fast.py:2865-2867) quantised for an MXFP8 cross_attn.q
 * (LINGBOT_LIN_MX, model_fast.py:1266-1269). */
int lbw_layernorm_affine_mx(const float* x, int m, int c, float eps, const float* weight, const float* bias,
                            void* data, void* scales, void* stream);
/* lbw_layernorm_affine_mx with the codes in element format fmt (LBW_MX_E4M3 or LBW_MX_E5M2). */
int lbw_layernorm_affine_mx_fmt(const float* x, int m, int c, float eps, const float* weight, const float* bias,
                                int fmt, void* data, void* scales, void* stream);

/* RMSNorm (+ 3-D RoPE) of projected rows: y = bf16(bf16(x * rsqrt(ss/c + eps)) * gamma), then,
 * if rope_cos != NULL, the interleaved-pair rotation with per-token angles of (frame, h, w).
 * x [m, c] bf16, ss [m] fp32, gamma [c] bf16; out rows out_row_off.. with row stride ldo.
 * rope tables: cos/sin [rope_frames*pf + grid_h*ph + grid_w*pw] fp32 laid out as
 * frame rows (pf = 22 pairs), then height rows (ph = 21), then width rows (pw = 21) for
 * head_dim 128; token t (global index tok0 + row) -> (t / (grid_h*grid_w), (t / grid_w) % grid_h, t % grid_w).
 * Replaces: WanRMSNorm (model.py:126-143), causal_rope_apply_rotation (model_fast.py:933-979),
 * qk_post.qk_norm_rope (kernels/qk_post.py:37-413). */
int lbw_rmsnorm_rope(const void* x, const float* ss, const void* gamma, int m, int c, float eps,
                     const float* rope_cos, const float* rope_sin, int rope_frames, int grid_h, int grid_w, int tok0,
                     void* out, long long ldo, int out_row_off, void* stream);
/* lbw_rmsnorm_rope of q and k of the same m tokens in ONE launch: q_out rows q_row_off.. (stride ldq) get q_raw's
 * normalised and rotated rows (ss_q, gamma_q), k_out rows k_row_off.. (stride ldk) k_raw's (ss_k, gamma_k); the
 * same RoPE tables and token numbering for both. Replaces: qk_post.qk_norm_rope (kernels/qk_post.py:37-413), which
 * normalises and rotates q and k together. */
int lbw_qk_rmsnorm_rope(const void* q_raw, const float* ss_q, const void* gamma_q, void* q_out, long long ldq,
                        int q_row_off, const void* k_raw, const float* ss_k, const void* gamma_k, void* k_out,
                        long long ldk, int k_row_off, int m, int c, float eps, const float* rope_cos,
                        const float* rope_sin, int rope_frames, int grid_h, int grid_w, int tok0, void* stream);
/* The same two with the rotation's arithmetic chosen: LBW_ROPE_FP32 (what the two above do: fp32 tables, products
 * and sums, one rounding to bf16) or LBW_ROPE_BF16, the reference's RoPE once a forward has seen a chunk of 4,096 or
 * more tokens (model_fast.py:1144-1148 set_bf16_rope_for_forward -> mark_bf16_rope :1000-1003, then
 * causal_rope_apply_rotation :933-979 with ROPE_DTYPE bf16 and the grids cast to bf16 :928-929): cos and sin
 * rounded to bf16, each product and each sum of the rotation rounded to bf16. */
#define LBW_ROPE_FP32 0
#define LBW_ROPE_BF16 1
int lbw_rmsnorm_rope_dt(const void* x, const float* ss, const void* gamma, int m, int c, float eps,
                        const float* rope_cos, const float* rope_sin, int rope_frames, int grid_h, int grid_w, int tok0,
                        void* out, long long ldo, int out_row_off, int rope_dtype, void* stream);
int lbw_qk_rmsnorm_rope_dt(const void* q_raw, const float* ss_q, const void* gamma_q, void* q_out, long long ldq,
                           int q_row_off, const void* k_raw, const float* ss_k, const void* gamma_k, void* k_out,
                           long long ldk, int k_row_off, int m, int c, float eps, const float* rope_cos,
                           const float* rope_sin, int rope_frames, int grid_h, int grid_w, int tok0, int rope_dtype,
                           void* stream);

/* ---- MXFP8 -------------------------------------------------------------------------------- */
/* Quantise bf16 x [rows, k] (k % 128 == 0) to E4M3 data [rows, k] and E8M0 scales in the tiled
 * layout (rows padded to 128, 512-byte atoms of 128 rows x 4 scales); optionally also the
 * dequantised bf16 values. Replaces: ffn_mx.prequantize_weight (kernels/ffn_mx.py:44-47) and
 * the in-kernel activation quantisation of ffn_mx.mm. */
int lbw_mx_quantize(const void* x, int rows, int k, void* data, void* scales, void* dequant, void* stream);

/* Element formats of the block-scaled path (OCP MX v1.0, one E8M0 scale per 32 elements along k). */
enum lbw_mx_format {
  LBW_MX_E4M3 = 0, /* MXFP8 E4M3: the reference's default (kernels/ffn_mx.py:18) */
  LBW_MX_E5M2 = 1, /* MXFP8 E5M2: LINGBOT_MX_FP8=float8_e5m2 (kernels/ffn_mx.py:8, :18) */
  LBW_MX_E2M1 = 2  /* MXFP4 E2M1: two elements per byte, element 2i in the low nibble (k % 256 == 0 for GEMMs);
                      not in the reference, the benchmark's block-scaled GEMM sweep asks for it */
};
/* lbw_mx_quantize in any lbw_mx_format: data [rows, k] bytes (E2M1: [rows, k / 2], packed), scales as above.
 * Replaces ffn_mx.prequantize_weight with LINGBOT_MX_FP8 (kernels/ffn_mx.py:8-18, :44-47). */
int lbw_mx_quantize_fmt(const void* x, int rows, int k, int fmt, void* data, void* scales, void* dequant, void* stream);

/* Block-scaled tcgen05 GEMMs (kind::mxf8f6f4, E4M3 x E4M3, E8M0 scale per 32 along K, fp32 accumulate).
 * a: codes [m, k] + tiled scales (rows padded to 128); w: codes [n, k] + tiled scales; k % 128 == 0,
 * n % 128 == 0. Replaces ffn_mx.mm (kernels/ffn_mx.py:159-182, nkilib matmul_mxfp8). */
/* Every epilogue rounds a w^T to bf16 before adding the bias, as ffn_mx.mm's bf16 result + bias does in the
 * reference (_mx_matmul, model_fast.py:1403-1410; _ffn_mx :1589-1610). */
/* out[m, n] = bf16(bf16(a w^T) + bias) (bias may be NULL). */
int lbw_mx_linear_fmt(const void* a, const void* a_scales, const void* w, const void* w_scales, const void* bias,
                      int m, int n, int k, int fmt, void* out, void* stream);
/* lbw_mx_linear_fmt in the element format lbw_mx_format fmt (E4M3 / E5M2: kind::mxf8f6f4; E2M1: kind::mxf4, K = 64
 * per MMA, k % 256 == 0); a and w as lbw_mx_quantize_fmt writes them. Replaces ffn_mx.mm (kernels/ffn_mx.py:159-182)
 * under LINGBOT_MX_FP8. */
int lbw_mx_linear(const void* a, const void* a_scales, const void* w, const void* w_scales, const void* bias, int m,
                  int n, int k, void* out, void* stream);
/* FFN up: GELU_tanh(bf16(a w^T) + bias) quantised to MXFP8 codes out[m, n] + tiled scales out_scales
 * (the down projection's A operand). Replaces ffn_mx.mm + ffn_epi.bias_gelu_pad (kernels/ffn_epi.py:15-37). */
int lbw_mx_linear_gelu(const void* a, const void* a_scales, const void* w, const void* w_scales, const void* bias,
                       int m, int n, int k, void* out, void* out_scales, void* stream);
/* lbw_mx_linear_gelu with operands and output codes in element format fmt (LBW_MX_E4M3 or LBW_MX_E5M2). */
int lbw_mx_linear_gelu_fmt(const void* a, const void* a_scales, const void* w, const void* w_scales, const void* bias,
                           int m, int n, int k, int fmt, void* out, void* out_scales, void* stream);
/* FFN down + gated residual: x[m, n] (fp32, in place) += bf16(a w^T + bias) * gate[n] (gate may be NULL).
 * Replaces ffn_mx.mm + bias and x + y * e5 (model_fast.py:1584-1611, :3110-3111). */
int lbw_mx_linear_residual(const void* a, const void* a_scales, const void* w, const void* w_scales,
                           const void* bias, int m, int n, int k, float* x, const float* gate, void* stream);
/* lbw_mx_linear_residual with operands in element format fmt (LBW_MX_E4M3 or LBW_MX_E5M2). */
int lbw_mx_linear_residual_fmt(const void* a, const void* a_scales, const void* w, const void* w_scales,
                               const void* bias, int m, int n, int k, int fmt, float* x, const float* gate,
                               void* stream);

/* The block's other Linears in MXFP8 (LINGBOT_LIN_MX=1, model_fast.py:1266-1269; _prequantize_linears_mx
 * :1442-1494 quantises each weight once, _mx_linear_forward :1413-1416 runs y = _mx_matmul(x) + b). */
/* q|k|v projection (w_qkv = [Wq; Wk; Wv] codes [3c, c] + scales): q_raw, k_raw [m, c] with row sums of squares
 * ss_q, ss_k [m] (cleared here) for the following RMSNorm, V rows v_row_off.. of v_out (row stride ldv).
 * The MXFP8 counterpart of lbw_qkv_proj (self_attn.q/k/v, model_fast.py:1733-1740). */
int lbw_mx_qkv_proj(const void* h, const void* h_scales, const void* w_qkv, const void* w_qkv_scales,
                    const void* b_qkv, int m, int c, void* q_raw, void* k_raw, float* ss_q, float* ss_k, void* v_out,
                    long long ldv, int v_row_off, void* stream);
/* lbw_mx_qkv_proj with operands in element format fmt (LBW_MX_E4M3 or LBW_MX_E5M2, LINGBOT_MX_FP8). */
int lbw_mx_qkv_proj_fmt(const void* h, const void* h_scales, const void* w_qkv, const void* w_qkv_scales,
                        const void* b_qkv, int m, int c, int fmt, void* q_raw, void* k_raw, float* ss_q, float* ss_k,
                        void* v_out, long long ldv, int v_row_off, void* stream);
/* out[m, n] = bf16(bf16(a w^T) + bias) with row sums of squares ss[m] (cleared here): cross_attn.q and, at the
 * first call, cross_attn.k on the text context (model_fast.py:2755-2798). */
int lbw_mx_linear_rowss(const void* a, const void* a_scales, const void* w, const void* w_scales, const void* bias,
                        int m, int n, int k, void* out, float* ss, void* stream);
/* lbw_mx_linear_rowss with operands in element format fmt (LBW_MX_E4M3 or LBW_MX_E5M2). */
int lbw_mx_linear_rowss_fmt(const void* a, const void* a_scales, const void* w, const void* w_scales, const void* bias,
                            int m, int n, int k, int fmt, void* out, float* ss, void* stream);
/* self_attn.o + gate + camera FiLM: x += bf16(bf16(a w^T) + bias) * gate, then x = (1 + s) * x + t (film_scale,
 * film_shift bf16 [m, n], both or neither). The MXFP8 counterpart of lbw_linear_residual (:3056-3089). */
int lbw_mx_linear_residual_film(const void* a, const void* a_scales, const void* w, const void* w_scales,
                                const void* bias, int m, int n, int k, float* x, const float* gate,
                                const void* film_scale, const void* film_shift, void* stream);
/* lbw_mx_linear_residual_film with operands in element format fmt (LBW_MX_E4M3 or LBW_MX_E5M2). */
int lbw_mx_linear_residual_film_fmt(const void* a, const void* a_scales, const void* w, const void* w_scales,
                                    const void* bias, int m, int n, int k, int fmt, float* x, const float* gate,
                                    const void* film_scale, const void* film_shift, void* stream);
/* Camera FiLM MLP layer: out = bf16(act(bf16(bf16(a w^T) + bias))) [+ addend, rounded to bf16], act = SiLU if silu
 * else identity. The MXFP8 counterpart of lbw_linear_act (cam_film, model_fast.py:2882-2891, :606-616). */
int lbw_mx_linear_act(const void* a, const void* a_scales, const void* w, const void* w_scales, const void* bias,
                      const void* addend, int silu, int m, int n, int k, void* out, void* stream);
/* lbw_mx_linear_act with operands in element format fmt (LBW_MX_E4M3 or LBW_MX_E5M2). */
int lbw_mx_linear_act_fmt(const void* a, const void* a_scales, const void* w, const void* w_scales, const void* bias,
                          const void* addend, int silu, int m, int n, int k, int fmt, void* out, void* stream);

/* ---- sequence-parallel K/V exchange (one process per GPU, same node, NVLink) ----------------
 * Replaces the all-gather of the new chunk's K/V shards into every rank's destination cache chunk
 * (wan/modules/model_fast.py:2066-2108 _gather_new, wan/distributed/tensor_parallel.py:106-139
 * all_gather_fn). Each rank owns one peer buffer (lbw_peer_buffer_create: cudaMalloc + CUDA IPC handle,
 * 64 bytes, exchanged by the caller) and opens the others' (lbw_peer_buffer_open). The exchange uses copy
 * engines and stream memory operations only: no SM is occupied, so it overlaps the attention of the cached
 * chunks. Buffer size: 4096 + 2 * local_rows * cols * 2 bytes. */
int lbw_peer_buffer_create(long long bytes, void** ptr, void* ipc_handle);
int lbw_peer_buffer_open(const void* ipc_handle, void** ptr);
/* owned = 1 for the caller's own buffer (freed), 0 for an opened peer buffer (unmapped). */
int lbw_peer_buffer_close(void* ptr, int owned);
/* The exchange's flag words: one LBW_SP_FLAG_BLOCK-byte block per rank in host memory that every rank of the node
 * maps (a POSIX shared-memory segment, say) and registers here: page-aligned, a whole number of pages. *dev = the
 * device address of `host` in this process. Block r holds ready[64] (byte 0), done[64] (byte 256) and a copy of
 * the gathered epoch (byte 512) of rank r. A rank's streams wait only on its own block, so a host thread can end
 * any of those waits by writing the awaited epoch there (the limit a stream memory operation does not have). */
#define LBW_SP_FLAG_BLOCK 1024
int lbw_host_flags_register(void* host, long long bytes, void** dev);
int lbw_host_flags_unregister(void* host);
/* One exchange = lbw_sp_kv_stage then lbw_sp_kv_gather with the same arguments (they may go on different
 * streams; the second on a stream ordered after the first). This rank's rows [rank*local_rows, +local_rows) of
 * k_dest / v_dest ([world*local_rows, ld] bf16, row stride ld elements, cols used) are sent to every peer, and
 * the peers' rows are received. bufs[p] = rank p's buffer as mapped in this process (bufs[rank] = own); flags =
 * the device address (lbw_host_flags_register) of rank 0's flag block, rank r's at flags + r*LBW_SP_FLAG_BLOCK.
 * epoch = 1, 2, ...: the number of this exchange on these buffers, the same on every rank.
 * stage: waits until every peer has finished reading the previous epoch, then copies this rank's rows into
 * its buffer. gather: announces them, waits until every peer has staged the same epoch (or the host writes the
 * epoch into this rank's flag block), pulls the peers' rows with copy engines (helper streams joined back into
 * `stream`), and, when all rows have landed, sets the 32-bit word at byte 512 of the own buffer to epoch (the
 * gate of lbw_chunk_attention_gated) and its copy in the own flag block. Replaces the K/V all-gather
 * (wan/modules/model_fast.py:2066-2108 _gather_new, wan/distributed/tensor_parallel.py:106-139). */
int lbw_sp_kv_stage(void* const* bufs, void* flags, int rank, int world, unsigned int epoch, void* k_dest,
                    void* v_dest, long long ld, int local_rows, int cols, void* stream);
int lbw_sp_kv_gather(void* const* bufs, void* flags, int rank, int world, unsigned int epoch, void* k_dest,
                     void* v_dest, long long ld, int local_rows, int cols, void* stream);

/* ---- Wan 2.1 VAE decoder (wan/modules/vae2_1.py) -------------------------------------------
 * Frames are stored channels-last with a one-pixel zero border: [frames][h + 2][w + 2][c] bf16 ("padded rows",
 * P = (h + 2)(w + 2) rows per frame). */
/* Causal 3-D / 2-D convolution as an implicit GEMM on the tcgen05 GEMM (CausalConv3d :16-35, the Resample Conv2d
 * :71-78 with kt = 1, the 1x1x1 shortcut). x: in_rows padded rows of c_in channels (c_in % 8 == 0) holding
 * kt - 1 history frames (the causal cache, or zeros) followed by `frames` input frames; w: [c_out, kt*kh*kw*ck]
 * bf16 with ck = c_in rounded up to a multiple of 64 (zero weights past c_in), K ordered (kt, kh, kw, c); out:
 * frames * P padded rows of c_out channels (c_out % 32 == 0), border rows
 * written as zeros; bias [c_out] and residual (same shape as out, added after rounding) may be NULL.
 * kt in {1, 3}, kh = kw in {1, 3}. */
int lbw_vae_conv(const void* x, long long in_rows, int c_in, const void* w, const void* bias, int c_out, int kt, int kh,
                 int kw, int frames, int h, int wd, const void* residual, void* out, void* stream);
/* lbw_vae_conv fused with the RMS_norm + SiLU that follows a ResidualBlock's first convolution (:189-192): out =
 * silu(y / max(||y||_2, 1e-12) * sqrt(c_real) * gamma) with y = bf16(conv + bias) over each row's c_out channels
 * (c_out <= 256: the row lies in one GEMM tile); gamma fp32 [c_out]; border rows zero. */
int lbw_vae_conv_rms(const void* x, long long in_rows, int c_in, const void* w, const void* bias, int c_out, int kt,
                     int kh, int kw, int frames, int h, int wd, const float* gamma, int c_real, void* out, void* stream);
/* out = RMS_norm(x) (x / max(||x||_2, 1e-12) * sqrt(c_real) * gamma, :38-53), then SiLU if silu != 0; one row
 * per voxel, c channels (c % 8 == 0, <= 512; channels past c_real are zero), gamma fp32 [c]. */
int lbw_vae_rms_silu(const void* x, long long rows, int c, int c_real, const float* gamma, int silu, void* out,
                     void* stream);
/* Nearest 2x upsampling in h and w ('nearest-exact', :56-62) of padded frames into padded frames of 2h x 2w. */
int lbw_vae_upsample2x(const void* x, int frames, int h, int w, int c, void* out, void* stream);
/* Resample upsample3d's frame interleave (:131-135): x [frames * frame_rows][2c] -> out [2 * frames * frame_rows][c],
 * frame 2f from channels [0, c), frame 2f + 1 from [c, 2c). */
int lbw_vae_time_interleave(const void* x, int frames, long long frame_rows, int c, void* out, void* stream);
/* AttentionBlock (:222-267) helpers: interior rows of padded frames -> compact token rows, and
 * out (padded) = resid + y (compact rows) inside, zero border. */
int lbw_vae_gather(const void* x, int frames, int h, int w, int c, void* out, void* stream);
int lbw_vae_scatter_add(const void* y, const void* resid, int frames, int h, int w, int c, void* out, void* stream);
/* fp32-output GEMM: out[m, n] = sum_k a[m, k] w[n, k] (the mid-block attention scores). */
int lbw_gemm_f32(const void* a, long long lda, const void* w, long long ldw, float* out, long long ldo, int m, int n,
                 int k, void* stream);
/* p[r, c] = softmax_c(scale * s[r, :n]) as bf16 for c < n, 0 for n <= c < n_pad. */
int lbw_softmax_rows(const float* s, long long lds, int rows, int n, int n_pad, float scale, void* p, long long ldp,
                     void* stream);
/* out[c][r] = x[r][c] (bf16). */
int lbw_transpose_bf16(const void* x, long long ldx, int rows, int cols, void* out, long long ldo, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* LBW_H_ */
