/*
 * sa3b200.h - C ABI of the B200 (sm_100a) Stable Audio 3 DiT denoiser path.
 *
 * Every entry point takes plain device pointers owned by the caller, sizes
 * and strides in ELEMENTS, and a CUDA stream (cudaStream_t passed as void*).
 * None of them allocates device memory, synchronises the host, or keeps
 * mutable state between calls except the device error word read by
 * sa3_get_device_error(). All launches are asynchronous on `stream` and can
 * be captured into CUDA graphs.
 *
 * Return value: SA3_OK (0) or a negative sa3_status. Argument errors are
 * detected on the host before anything is launched.
 *
 * Layout convention ("token rows"): activations are row-major 2-D views
 * [rows, features]; a row is one token, features hold all heads
 * (head h occupies columns [h*head_dim, (h+1)*head_dim)). This is the layout
 * nn.Linear produces, so projections feed attention without transposes.
 */
#ifndef SA3B200_H
#define SA3B200_H

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  SA3_OK = 0,
  SA3_ERR_ARG = -1,         /* bad size / null pointer / inconsistent arguments */
  SA3_ERR_ALIGN = -2,       /* pointer or stride violates the 16-byte rule */
  SA3_ERR_DTYPE = -3,       /* dtype combination not supported */
  SA3_ERR_LAUNCH = -4,      /* CUDA launch or driver call failed */
  SA3_ERR_UNSUPPORTED = -5, /* shape outside what the kernels implement */
} sa3_status;

/* device error word codes (low byte) */
#define SA3_DEVERR_TIMEOUT 1

/* element types */
#define SA3_DT_BF16 0
#define SA3_DT_F16 1
#define SA3_DT_E4M3 2
#define SA3_DT_F32 3

/* ------------------------------------------------------------------ misc */

/* Library version (major*10000 + minor*100 + patch). */
int sa3_version(void);

/* Reads and clears the device error word of the current device (0 = no
 * kernel reported a timed-out wait). Synchronises the device. */
int sa3_get_device_error(int* err);

/* ------------------------------------------------------------- GEMM (a3, a4)
 *
 * C[M, N] = epilogue( (A[M, K] . B[N, K]^T) * a_scale * b_scale[n] + bias[n] )
 *
 * Replaces the nn.Linear calls of the DiT trunk:
 *   Attention.to_qkv / to_q / to_kv / to_out  (stable_audio_3/models/transformer.py:547-560)
 *   GLU.proj + SiLU gate                        (transformer.py:421-444)
 *   FeedForward linear_out                      (transformer.py:485)
 * with the adaLN gate + residual of TransformerBlock.forward
 * (transformer.py:1027-1029, 1047-1049) fused into the epilogue.
 *
 * A and B are K-major (B is the nn.Linear weight [out, in]). ab_dtype is
 * SA3_DT_BF16 (tcgen05 kind::f16) or SA3_DT_E4M3 (kind::f8f6f4).
 * a_scale: device fp32 scalar or NULL (1). b_scale: device fp32 [N] or NULL.
 * bias: device fp32 [N] or NULL. lda/ldb/ldc in elements; A, B rows must be
 * 16-byte aligned (lda*elt and ldb*elt multiples of 16).
 */
#define SA3_EPI_STORE 0          /* C = acc (bf16) */
#define SA3_EPI_SILU 1           /* C = silu(acc) */
#define SA3_EPI_SWIGLU 2         /* B rows interleaved in blocks of 128 [x|gate]; C[:, N/2] = x*silu(gate) */
#define SA3_EPI_GATED_RESIDUAL 3 /* C = residual + acc * sigmoid(1 - gate[batch(row), n]) */
#define SA3_EPI_RESIDUAL 4       /* C = residual + acc */
#define SA3_EPI_QK_NORM 5        /* C = acc, then per 64-column head: RMSNorm(gamma of its column group) and
                                    RoPE on dims 0..31 where enabled (fuses sa3_qk_norm_rope into to_qkv /
                                    to_q / to_kv; Attention.apply_qk_layernorm + apply_rotary_pos_emb,
                                    transformer.py:589-595, 302-322, 755-781) */

typedef struct {
  int kind;                 /* SA3_EPI_* */
  const float* bias;        /* [N] fp32 or NULL */
  const void* residual;     /* C's dtype (bf16, or fp32 / fp16 below), row stride ld_residual; may alias C */
  long long ld_residual;
  const float* gate;        /* fp32 gate rows: batch b reads gate + b*ld_gate */
  long long ld_gate;
  int rows_per_batch;       /* batch(row) = row / rows_per_batch when row_batch is NULL */
  const int* row_batch;     /* optional int32 [M]: batch index of each row */
  float* amax_out;          /* optional: atomic max of |stored value| (non-negative, caller zeroes) */
  int seg_in;               /* output row remap: if > 0, out_row = (m / seg_in) * seg_out + seg_offset + m % seg_in */
  int seg_out;
  int seg_offset;
  int c_f32;                /* nonzero: C and residual are fp32 (the fp32 residual stream), else bf16 */
  /* SA3_EPI_QK_NORM only: columns form groups of qk_group_width (a multiple of 64); group g's heads are
     RMS-normalised with qk_gamma[g] (64 fp32, 16-byte aligned; NULL = left as is) and, if bit g of
     qk_rope_mask is set, rotated at position row_pos[m] (or m % rows_per_batch) with the cos/sin
     table of sa3_qk_norm_rope. */
  const float* qk_gamma[8];
  int qk_group_width;
  unsigned qk_rope_mask;
  float qk_eps;
  const float* cos_sin;
  int max_pos;
  const int* row_pos;
  /* optional int32 [M]: output (and residual) row of GEMM row m; overrides seg_*. Packs variable-length
     sequences (project_in, the local-conditioning add) into the token-row stream. */
  const int* out_row_map;
  /* SA3_EPI_QK_NORM with more than 8 groups (the cross-attention K/V projections of every block in one
     GEMM): when qk_gamma_table is non-NULL it replaces qk_gamma. Groups g < qk_table_groups are
     RMS-normalised with the 64 fp32 at qk_gamma_table + 64 g (16-byte aligned); later groups are left as
     is. qk_rope_mask must be 0 in this mode. Zero-initialised callers get the 8-group behaviour. */
  const float* qk_gamma_table;
  int qk_table_groups;
  /* nonzero (with c_f32 zero): C and residual are fp16, the half-precision residual stream. Supported for
     SA3_EPI_STORE / SILU (any row remap) and the residual kinds; an in-place residual (residual == C, same row
     stride, no row remap, no amax_out) is added by a TMA reduce-add in fp16: the L2 adds fp16(acc) to C with
     round-to-nearest. Other combinations return SA3_ERR_UNSUPPORTED. */
  int c_f16;
} sa3_epilogue;

int sa3_gemm(const void* A, const void* B, void* C, int M, int N, int K, long long lda, long long ldb,
             long long ldc, int ab_dtype, const float* a_scale, const float* b_scale, const sa3_epilogue* epi,
             void* stream);

/* ---------------------------------------------- GPTQ int4 weight-only linear (a3, a4)
 *
 * C = epilogue(A . W^T) with W stored 4-bit: replaces the same nn.Linear calls as
 * sa3_gemm (transformer.py:547-560, 432, 485) for GPTQ checkpoints (asymmetric,
 * group size gs, act-order). The reference has no quantized code; the layout below
 * is this library's, produced from the usual GPTQ tensors (qweight [K/8, N],
 * qzeros [G, N/8], fp16 scales [G, N], g_idx [K]) by sa3_b200.gptq.repack:
 *   perm int32 [K]    : input channels sorted by group (stable argsort of g_idx);
 *                       A must hold x[:, perm] (sa3_permute_cols)
 *   qw   int32 [N, K/8] : word (n, w) = q[n, perm[8w + j]] in bits [4j, 4j+4), LSB first
 *   sz   fp32  [G, 2N]  : row g = [ s[g, :] | z[g, :] * s[g, :] ]
 * W[n, k'] = (q - z) * s computed as fma(q, s, -z*s) in fp32 (exact), rounded once to bf16
 * in shared memory, multiplied on tcgen05 (kind::f16) with fp32 accumulation.
 * A bf16 [M, K] (lda); K % gs == 0, gs % 64 == 0, N % 256 == 0. Epilogue as sa3_gemm
 * (a_scale / b_scale do not apply).
 */
int sa3_gptq_gemm(const void* A, const void* qw, const float* sz, void* C, int M, int N, int K, long long lda,
                  long long ldc, int group_size, const sa3_epilogue* epi, void* stream);

/* Dequantise the packed GPTQ weight to bf16 W [N, K] (row n contiguous over the sorted channels),
 * with the exact arithmetic of sa3_gptq_gemm's shared-memory stage. */
int sa3_gptq_dequant(const void* qw, const float* sz, void* out, int N, int K, int group_size, void* stream);

/* Dequantise the packed GPTQ weight to bf16 W [N, K] (row stride ldo) in the ORIGINAL input-channel
 * order, i.e. the dense weight of the nn.Linear the layer replaces (transformer.py:547-560, 432, 485):
 * W[n, k] = (q - z) * s of sorted position inv_perm[k] (inv_perm = the inverse of perm), with the exact
 * arithmetic of sa3_gptq_gemm. For large M, dequantising once per call and running sa3_gemm (bf16) on the
 * unpermuted activations replaces both the act-order gather and the per-tile dequantisation. */
int sa3_gptq_dequant_orig(const void* qw, const float* sz, const int* inv_perm, void* out, int N, int K,
                          long long ldo, int group_size, void* stream);

/* out[r, j] = x[r, perm[j]] for a bf16 [rows, K] view (the act-order gather of GPTQ inputs). */
int sa3_permute_cols(const void* x, const int* perm, void* out, int rows, int K, long long ldx, long long ldo,
                     void* stream);

/* ---------------------------------------------- glue: norms / modulation (a7, a9)
 *
 * y[r, :] = RMSNorm(x[r, :]) * gamma * (1 + scale[b, :]) + shift[b, :]
 *   RMSNorm  : stable_audio_3/models/transformer.py:392-410 (F.rms_norm)
 *   modulate : transformer.py:1020-1026, 1043-1045 (x * (1 + scale) + shift)
 * b = batch(r) as in sa3_epilogue. `mod` is NULL for a plain RMSNorm
 * (cross_attend_norm, transformer.py:1033); otherwise scale of batch b is
 * mod + b*ld_mod + scale_off and shift is mod + b*ld_mod + shift_off (fp32).
 * gamma: fp32 [D] or NULL.
 * mode SA3_NORM_WRITE writes y as out_dtype (BF16 or E4M3; E4M3 multiplies by
 *   r = 448 / max(*quant_amax, 1e-12) first and saturates, and, if scale_out
 *   is non-NULL, stores s = max(*quant_amax, 1e-12) / 448 there for the
 *   consuming GEMM's a_scale).
 * mode SA3_NORM_AMAX writes nothing and atomically maxes |y| into *amax_out.
 * x is bf16, fp16 or fp32 (x_dtype) [rows, D]; D must be a multiple of 8, rows 16-byte aligned.
 * row_r (optional, fp32 [rows]): the AMAX pass stores each row's 1/rms there and the WRITE pass of the
 *   same x reads it instead of recomputing it, which turns that pass into an elementwise stream (same
 *   output). The AMAX pass with row_r must have run on the same stream before such a WRITE pass. The
 *   AMAX pass stores it for fp16 / fp32 x with D = 1024, 1536 or 2048 (16-byte aligned gamma /
 *   modulation rows); the WRITE pass uses it for fp16 x with at most two uniform modulation batches
 *   (row_batch NULL) or no modulation. Other calls ignore row_r.
 */
#define SA3_NORM_WRITE 0
#define SA3_NORM_AMAX 1
int sa3_rmsnorm_modulate(const void* x, int x_dtype, void* out, int rows, int D, long long ldx, long long ldo,
                         const float* gamma,
                         float eps, const float* mod, long long ld_mod, int scale_off, int shift_off,
                         int rows_per_batch, const int* row_batch, int mode, int out_dtype,
                         const float* quant_amax, float* scale_out, float* amax_out, float* row_r,
                         void* stream);

/* One launch for an FP8 (or bf16) norm of the fp16 stream: the AMAX pass and the WRITE pass of
 * sa3_rmsnorm_modulate with row_r, joined by a grid-wide barrier. *amax accumulates max|y| as the AMAX
 * pass does (start it at 0); out receives y (e4m3 scaled by 448 / max(*amax, 1e-12), or bf16) and
 * *scale_out (if non-NULL) the dequantisation scale. row_r: fp32 [rows] scratch. barrier: two uint32
 * (8-byte aligned), zero before the first call, left ready for the next; one stream at a time may use
 * them. The single launch serves fp16 x with D = 1536 and at most two uniform modulation batches (or
 * none); other calls issue the two passes. Either way the bytes equal the two passes'. Every block of
 * the launch must be resident at once (the grid is capped at the kernel's occupancy); the barrier's
 * wait gives up after about a second with device error site 95. */
int sa3_rmsnorm_quant_fused(const void* x, int x_dtype, void* out, int rows, int D, long long ldx, long long ldo,
                            const float* gamma, float eps, const float* mod, long long ld_mod, int scale_off,
                            int shift_off, int rows_per_batch, const int* row_batch, int out_dtype, float* amax,
                            float* scale_out, float* row_r, unsigned int* barrier, void* stream);

/* Per-tensor dynamic FP8 quantisation: out = e4m3(x * r), r = 448/max(*amax,1e-12);
 * the dequantisation scale s = max(*amax,1e-12)/448 is stored to *scale_out when non-NULL. If amax_out is non-NULL, the
 * kernel only computes max|x| into it (no write). x is bf16. */
int sa3_quantize_e4m3(const void* x, void* out, int rows, int cols, long long ldx, long long ldo,
                      const float* amax, float* scale_out, float* amax_out, void* stream);

/* Element type conversion of a row-major [rows, cols] view: fp32 <-> bf16
 * (round to nearest even). cols must be a multiple of 8, rows 16-byte aligned.
 * src_rows (optional int32 [rows]): output row r reads input row src_rows[r].
 * Used to hand the fp32 residual stream to a bf16 GEMM operand (project_out,
 * transformer.py:1267). */
int sa3_convert(const void* x, int x_dtype, void* out, int out_dtype, int rows, int cols, long long ldx,
                long long ldo, const int* src_rows, void* stream);

/* ---------------------------------------------- glue: qk-norm + partial RoPE (a5, a6)
 *
 * In place on up to 4 head groups of a token-row buffer (e.g. q, k, q_diff,
 * k_diff inside the fused to_qkv output). For every row r and head h of
 * group g (columns col_off[g] + h*64 .. +63):
 *   t = RMSNorm_64(t) * gamma_g            (Attention.apply_qk_layernorm, transformer.py:589-595, eps 1e-6)
 *   if rope[g]: t[0:32] = t*cos + rotate_half(t)*sin at position pos(r)
 *                         (apply_rotary_pos_emb / rotate_half, transformer.py:296-322; fp32)
 * pos(r) = row_pos[r] if row_pos else r % rows_per_batch.
 * cos_sin: fp32 table [max_pos, 32]: cols 0..15 cos(pos*inv_freq[i]),
 *          cols 16..31 sin(pos*inv_freq[i])  (RotaryEmbedding, transformer.py:239-294).
 * head_dim must be 64, rot_dim 32.
 */
int sa3_qk_norm_rope(void* buf, int rows, long long ld, int heads, int ngroups, const int* col_off,
                     const float* const* gamma, const int* rope, float eps, const float* cos_sin, int max_pos,
                     int rows_per_batch, const int* row_pos, void* stream);

/* ---------------------------------------------- attention (a1, a2, a11)
 *
 * out = softmax(q k^T * scale + band) v           (differential: minus the same with q2, k2)
 * Replaces flash_attn_func / flash_attn_varlen_func(..., window_size=(wl, wr))
 * as called from Attention.apply_attn (stable_audio_3/models/transformer.py:641-666),
 * the differential combine out - out_diff (transformer.py:790-795) and the
 * non-windowed cross-attention (transformer.py:1031-1035).
 *
 * Band (flash-attn convention, bottom-right aligned): key j of a sequence is
 * visible to query i iff  i + (Lk - Lq) - wl <= j <= i + (Lk - Lq) + wr;
 * a negative wl / wr means unbounded on that side.
 * Sequences: if cu_seqlens_q is NULL, sequence b has rows [b*Lq, (b+1)*Lq)
 * (same for k with Lk); otherwise rows [cu[b], cu[b+1]) (int32, device).
 * q, k, v, q2, k2, v2, out are token-row buffers with the given row strides;
 * head h sits at columns h*64 of each. q2/k2 NULL = not differential;
 * v2 NULL = the second stream reuses v (the DiT's differential attention),
 * otherwise it reads its own values (the SAME-L plugin op below).
 * dtype: SA3_DT_BF16 or SA3_DT_F16 (operands, P and output). head_dim must be 64.
 * amax_out (optional): atomic max of |stored output| for a following FP8 quantisation.
 */
int sa3_attention(const void* q, const void* k, const void* v, const void* q2, const void* k2, const void* v2,
                  void* out,
                  const int* cu_seqlens_q, const int* cu_seqlens_k, int batch, int max_seqlen_q, int max_seqlen_k,
                  int total_q, int total_k, int heads, int head_dim, long long ldq, long long ldk, long long ldv,
                  long long ldo, int window_left, int window_right, float softmax_scale, int dtype,
                  float* amax_out, void* stream);

/* ---------------------------------------------- allocation-free FP8 linear
 *
 * No counterpart in the reference: an addition for callers that cannot
 * allocate device memory, such as a TensorRT plugin's enqueue (TensorRT
 * plans all memory ahead and an enqueue must not allocate), or a host with a
 * fixed device-memory budget that cannot risk the implicit device
 * synchronisation of cudaMalloc mid-stream.
 *
 * out[M, N] (bf16) = (e4m3(x * r_x) * s_x) . (w * w_scale[n])^T + bias[n], i.e.
 * the same FP8 linear as sa3_quantize_e4m3 (max|x| pass, quantise pass) followed
 * by sa3_gemm, but its scratch (max|x|, s_x and the M*K-byte e4m3 copy of x)
 * lives in a file-scope device array of 16 MiB, so the call allocates nothing.
 * x: bf16 [M, K] (row stride ldx >= K, a multiple of 8, 16-byte aligned);
 * w: e4m3 [N, K] (ldw >= K, a multiple of 16, 16-byte aligned); w_scale fp32
 * [N] (or NULL); bias fp32 [N] (or NULL); ldo >= N; K a multiple of 16. Every
 * argument error is returned before anything is launched or the scratch is
 * touched.
 * Limit: M * K <= SA3_FP8_NOALLOC_MAX_ELEMS, else SA3_ERR_UNSUPPORTED with
 * nothing launched. The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress) and keeps it for the process, so make that
 * first call before any stream capture; a device reset (cudaDeviceReset) is
 * not supported afterwards. The array is shared by every call and keeps the
 * last call's contents; calls that overlap on the GPU race on it.
 */
#define SA3_FP8_NOALLOC_MAX_ELEMS ((16LL << 20) - 256)
int sa3_fp8_linear_noalloc(const void* x, const void* w, const float* w_scale, const float* bias, void* out, int M,
                           int N, int K, long long ldx, long long ldw, long long ldo, void* stream);

/* ---------------------------------------------- SWA plugin op (a15, f3)
 *
 * The operator of the TensorRT plugin samel::diff_attn_swa
 * (optimized/tensorRT/scripts/diff_attn_nocast_plugin.py:14-41, kernel
 * triton_swa_v2.py:94-119): q_bat, k_bat, v_bat are [B, N, 2H, d] with the two
 * differential streams stacked on the head axis; out [B, N, H, d] =
 * attn(heads 0..H-1) - attn(heads H..2H-1), each with its own q/k/v, window
 * |i - j| <= window, scale d^-1/2. Writes into the caller-owned out on stream.
 * dtype SA3_DT_BF16 or SA3_DT_F16 (fp32 callers convert first).
 */
int sa3_diff_attn_swa(const void* q_bat, const void* k_bat, const void* v_bat, void* out, int dtype, int batch,
                      int seqlen, int num_heads, int head_dim, int window, void* stream);

/* ---------------------------------------------- sequence split: max over ranks through peer memory (e)
 *
 * Replaces the 4-byte NCCL all-reduce (MAX) of the per-tensor FP8 activation amax
 * that the sequence-split step makes at every quantisation point (the reference
 * has no sequence split; the split is this library's, see sa3_b200/seqsplit.py).
 * Each rank allocates a mailbox (sa3_peer_box_alloc, sa3_peer_box_bytes() bytes,
 * zeroed) and shares it with the other ranks of the node through a CUDA IPC
 * handle (sa3_ipc_get_handle / sa3_ipc_open_handle, sa3_ipc_handle_bytes()
 * bytes). sa3_peer_max(value, boxes, rank, world, stream) then replaces *value
 * (fp32, device) with its maximum over the world ranks: boxes[r] is rank r's
 * mailbox as this process addresses it (its own allocation for r == rank, the
 * opened IPC pointer otherwise). One warp stores (epoch, value) into every
 * rank's mailbox over NVLink and waits, bounded by about a second, for every
 * rank's word of the same epoch; on timeout it records device error site 90 and
 * keeps the local value. Every rank must make the same calls in the same order,
 * each rank on its own GPU of one node with peer access (never two ranks on one
 * GPU: their kernels wait on each other). world <= SA3_PEER_MAX_RANKS.
 */
#define SA3_PEER_MAX_RANKS 8
#define SA3_PEER_SLOTS 4
int sa3_peer_box_bytes(void);
int sa3_peer_box_alloc(void** box);
int sa3_peer_box_free(void* box);
int sa3_ipc_handle_bytes(void);
int sa3_ipc_get_handle(void* ptr, void* handle);
int sa3_ipc_open_handle(const void* handle, void** ptr);
int sa3_ipc_close_handle(void* ptr);
int sa3_peer_max(float* value, void* const* boxes, int rank, int world, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SA3B200_H */
