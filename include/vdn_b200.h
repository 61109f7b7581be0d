/*
 * vdn_b200.h - C ABI of libvdn_b200.so, the sm_100a hot path of the VDN-H3 hybrid
 * attention block (hyukudan/ComfyUI-Kirei-VDN-H3 v0.3.3).
 *
 * Conventions for every entry point:
 *   - pointers are CUDA device pointers (row-major, pitches in elements), sizes are
 *     plain ints; `stream` is a cudaStream_t passed as void*; all work is stream-ordered;
 *   - the return value is a status: 0 ok, -1 invalid argument, -2 unsupported geometry,
 *     -3 TMA tensor-map encoding failed, -4 launch failed, -5 misaligned pointer/pitch,
 *     -6 problem larger than a fixed device scratch area;
 *   - `dev_err` (where present) is a device int that receives the first kernel abort
 *     code (1..4: a bounded wait timed out); the host checks it once per forward;
 *   - bf16 = __nv_bfloat16, fp8 = e4m3 (float8_e4m3fn), int8 = signed char.
 *
 * The reference is pure Python/torch; each function below names the reference code it
 * replaces (file:line inside the reference project).  The package's Python host binds every
 * entry point with ctypes (argument types declared per function, int status returned),
 * mapping the status codes onto the exceptions the reference raises.
 */
#ifndef VDN_B200_H
#define VDN_B200_H

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- projections ---- */

/* C = epilogue(A * B^T).  kind: 0 bf16, 1 fp8 e4m3, 2 int8.  A: [M, K] (pitch lda), or
 * split along K: A for k < k_split, A2 (pitch lda2) for the rest (A2 = NULL: one source).
 * B: [N, K] (pitch ldb).  out_kind: 0 bf16, 1 fp32, 2 raw int32 (int8 only).
 * epilogue: v = acc * alpha * dev_scale0 * dev_scale1 * row_scale[m] * col_scale[n]
 *           (+ col_bias[n]) (sigmoid if act == 1) (+ addend[m, n] bf16).
 * Replaces: hybrid.py:263 and :535 (ComfyUI qkv_proj / out_proj linears),
 *           projection.py:259-268 (project), fp8.py:239-266 (_scaled_mm),
 *           projection.py:243-256 (ck.int8_linear), branch.py:754-758 (output gate). */
int vdn_gemm(int kind, const void* A, long long lda, const void* A2, long long lda2, long long k_split,
             const void* B, long long ldb, void* C, long long ldc, int out_kind, int M, int N, int K,
             float alpha, const float* dev_scale0, const float* dev_scale1, const float* row_scale,
             const float* col_scale, const float* col_bias, int act, const void* addend, long long ld_add,
             int* dev_err, void* stream);

/* vdn_gemm with a grouped-K A operand: A is `groups` slabs of [M, kg] (rows lda elements
 * apart, slabs group_stride elements apart) read in order as one [M, groups*kg] operand;
 * kg must be a multiple of the k-block (64 bf16, 128 fp8/int8).  Used for the row-split
 * output projection of the head-sharded block, reading the all-to-all receive buffer
 * [ranks][rows][2*heads_per_rank*head_dim] in place.
 * No reference counterpart: the reference runs one GPU per block (hybrid.py:534-540 is the
 * projection this feeds). */
int vdn_gemm_grouped_k(int kind, const void* A, long long lda, long long group_stride, int groups, int kg,
                       const void* B, long long ldb, void* C, long long ldc, int out_kind, int M, int N,
                       float alpha, const float* dev_scale0, const float* dev_scale1, const float* row_scale,
                       const float* col_scale, const float* col_bias, int act, const void* addend,
                       long long ld_add, int* dev_err, void* stream);

/* Fused QKV projection of x [S, hidden] against [W_qkv; W_side] ([3*inner + n_aux, hidden]):
 * raw q/k/v -> qkv_out [S, 3*inner] bf16; RMSNorm(q), RMSNorm(k) per head with weights
 * norm_w [2, head_dim] fp32 -> qk_norm [S, 2*inner] bf16; side columns -> aux_out [S, n_aux] fp32.
 * kind / scales as in vdn_gemm (int8: row_scale per token, col_scale per channel).
 * Replaces: hybrid.py:260-268 (_qkv), hybrid.py:271-273 (q_norm / k_norm, rope_freqs=None),
 *           hybrid.py:520-522 (gate logits), branch.py:736 (beta), :743-751 (alpha down),
 *           :755 (output-gate down).  q_act (optional): the branch's q features of rows
 * [act_row0, act_row0 + act_rows) -- silu(bf16 q) L2-normalised per head, stored
 * [frame][head][token][head_dim] with act_tpf tokens per frame (kernels.py:47-51 and the FHSD
 * permute of branch.py:672-689).  act_row0 counts from this call's first row (it may be
 * negative when the call covers a block of rows starting inside the branch rows). */
int vdn_qkv_gemm(int kind, const void* x, long long ldx, const void* w, long long ldw, int S, int hidden,
                 int inner, int n_aux, int head_dim, const float* norm_w, float eps, float alpha,
                 const float* dev_scale0, const float* dev_scale1, const float* row_scale,
                 const float* col_scale, void* qkv_out, long long ld_qkv, void* qk_norm, long long ld_norm,
                 float* aux_out, long long ld_aux, void* q_act, int act_row0, int act_rows, int act_tpf,
                 int* dev_err, void* stream);

/* Per-row symmetric int8 (scale = max(amax/127, 1e-12), round half to even).
 * src_kind: 0 bf16, 1 fp32.  Replaces: projection.py:74-97 (TensorWiseINT8 quantisation,
 * here without ConvRot: the config-2 scheme). */
int vdn_quant_int8_rows(int src_kind, const void* x, long long ldx, int rows, int K, void* q, long long ldq,
                        float* scale, void* stream);

/* ConvRot int8 rows: each 256-wide group of a bf16 row [rows, K] is rotated by R/16, R the
 * fourth Kronecker power of the order-4 regular Hadamard matrix J - 2I (symmetric and
 * orthogonal up to 1/16), then quantised per row as vdn_quant_int8_rows.  Applied to the
 * activation rows and to the weight rows alike, it leaves x W^T unchanged.  group must be
 * 256; K % 256 == 0, K <= 32768; 16-byte aligned x rows, 8-byte aligned q rows.
 * Replaces: the ConvRot rotation + TensorWiseINT8 quantisation that comfy-kitchen's
 * ck.int8_linear / QuantizedTensor.from_float(convrot=True, convrot_groupsize=256) perform
 * for projection.py:74-97 and :243-256 (comfy-kitchen is outside the reference tree, so its
 * exact Hadamard ordering and activation scaling are not pinned). */
int vdn_quant_int8_rows_convrot(const void* x, long long ldx, int rows, int K, int group, void* q, long long ldq,
                                float* scale, void* stream);

/* Per-tensor e4m3 (scale = max(amax/448, 1e-12)); work: one fp32 device scalar.
 * Replaces: fp8.py:108-133 (quantize_activation, per_tensor=True). */
int vdn_quant_fp8_tensor(int src_kind, const void* x, long long ldx, int rows, int K, void* q, long long ldq,
                         float* work, float* scale_out, void* stream);

/* The two halves of vdn_quant_fp8_tensor: vdn_fp8_amax zeroes and fills amax (device fp32);
 * vdn_fp8_cast quantises with a given amax and writes the scale.  Between them the
 * head-sharded block all-reduces amax (MAX) so a row-split projection uses the scale of
 * the whole tensor.  Replaces: fp8.py:99-133 (per_tensor=True), split in two steps; the
 * split itself has no reference counterpart. */
int vdn_fp8_amax(int src_kind, const void* x, long long ldx, int rows, int K, float* amax, void* stream);
int vdn_fp8_cast(int src_kind, const void* x, long long ldx, int rows, int K, const float* amax, void* q,
                 long long ldq, float* scale_out, void* stream);

/* FP8 projection that allocates nothing (no counterpart in the reference: an addition for
 * callers that cannot allocate device memory while they run, e.g. code running inside a
 * memory arena it does not own or a host that hands the library a fixed device budget).
 * out[M, N] bf16 = x[M, K] bf16 * W^T with x quantised per tensor to e4m3 in the library's
 * own file-scope device scratch array; W [N, K] e4m3, w_scale one fp32 device scalar.
 * Limit: M * K <= 16,777,216 (else -6, nothing done); K % 16 == 0; ldx, ldw >= K and
 * ldo >= N (else -1).  The array (~16 MiB) stays resident on every GPU that loads the
 * library; the first call on a device looks up its address (make it before any stream
 * capture); calls that overlap on the GPU race. */
int vdn_fp8_linear_noalloc(const void* x, long long ldx, int M, int K, const void* w_fp8, long long ldw, int N,
                           const float* w_scale, void* out, long long ldo, int* dev_err, void* stream);

/* ---------------------------------------------------------------- window softmax -- */

/* Exact block-sparse window softmax attention with the per-token head gate fused.
 * q, k, v: [S, H*D] bf16 views (pitches ld_q/ld_k/ld_v); q, k already RMS-normalised.
 * frame_lo/frame_hi [F]: clamped visible key-frame range; items/tile_off/qtile/ktile: host
 * plan (window.py in the package); qtile [n_qtiles][2] = per 128-row half (first row << 8) | rows,
 * rows <= 128, 0 for an empty half whose first row is still valid (null: tile t covers rows
 * [256 t, 256 t + 256)).  out [S, ld_out] bf16 at columns h*D.
 * gate_logits [S, ld_gate] fp32 (column gate_col0 + h) + gate_bias [H]: optional.
 * work_counter: one device int (zeroed on the stream by the call) through which the
 * persistent CTAs claim work items; calls sharing it must not overlap on the GPU.
 * Replaces: window.py:277-313 (window_softmax_grouped), window.py:327-344 (mask),
 *           window.py:694-861 (flex / FA2 / FA4 backends), hybrid.py:518-528 and
 *           softmax_kernels.py:8-37 (gate and flatten). */
int vdn_window_attention(const void* q, long long ld_q, const void* k, long long ld_k, const void* v,
                         long long ld_v, int S, int H, int D, int video_start, int video_end, int num_frames,
                         int tokens_per_frame, int anchor_rows, int anchor_cols, float scale,
                         const int* frame_lo, const int* frame_hi, const int* items, int n_items,
                         const int* tile_off, const int* qtile, const int* ktile, void* out, long long ld_out,
                         const float* gate_logits, long long ld_gate, int gate_col0, const float* gate_bias,
                         int* work_counter, int* dev_err, void* stream);

/* ---------------------------------------------------------------- VDA branch ------ */

/* Depthwise kh x kw conv per frame on the (gh, gw) grid, zero padding; out bf16.
 * Replaces: branch.py:469-471, runtime.py:329-333 (F.conv2d groups=channels). */
int vdn_spatial_conv(const void* in, long long ld_in, const float* w, int kh, int kw, int F, int gh, int gw,
                     int C, void* out, long long ld_out, void* stream);

/* Temporal depthwise conv (taps 5, zero pad; taps 0 = none), SiLU, optional L2 over D,
 * output FHSD [F, H, T, D] bf16.  Replaces: kernels.py:99-162 (_tconv_act_kernel),
 * kernels.py:59-68 (temporal_shift_eager), kernels.py:47-51 (activate). */
int vdn_temporal_act(const void* in, long long ld_in, const float* w, int taps, int F, int T, int H, int D,
                     int l2norm, void* out, void* stream);

/* The two above in one pass: depthwise 5x5 spatial conv (bf16-rounded), 5-tap temporal conv,
 * SiLU, optional L2 over D, FHSD output [F, H, gh*gw, D] bf16, with no intermediate in
 * memory.  w_sp [H*D, 25], w_tm [H*D, 5] fp32; in 16-byte aligned, ld_in % 8 == 0.
 * -2 unless kh = kw = taps = 5 and D is 64 or 128.  Replaces: branch.py:443-480
 * (conv_features), runtime.py:311-348 (_feature_one), kernels.py:99-129. */
int vdn_conv_features(const void* in, long long ld_in, const float* w_sp, int kh, int kw, const float* w_tm,
                      int taps, int F, int gh, int gw, int H, int D, int l2norm, void* out, void* stream);

/* alpha [F, H, D] = exp(-exp(A_log) * softplus(W_up mean_t(down) + dt_bias)), down being the
 * per-row x W_down^T columns.  Replaces: branch.py:483-491 (alpha_gate), :743-751. */
int vdn_alpha_gate(const float* down, long long ld_down, int F, int T, int R, const float* w_up,
                   const float* dt_bias, const float* a_log, int H, int D, float* alpha, void* stream);

/* A = sym((beta K)^T K), B = (beta V)^T K per frame and head, beta = sigmoid(logit).
 * Replaces: branch.py:197-282 (frame_statistics). */
int vdn_frame_stats(const void* K, const void* V, int F, int H, int T, int D, const float* beta_logits,
                    long long ld_beta, int beta_col0, float* A, float* B, void* stream);

/* Tensor-core frame statistics for head_dim 128 (same contract as vdn_frame_stats):
 * A = (beta K)^T K, B = (beta V)^T K as tcgen05 MMAs over 128-token chunks.
 * Replaces: branch.py:197-282 (frame_statistics). */
int vdn_frame_stats_tc(const void* K, const void* V, int F, int H, int T, const float* beta_logits,
                       long long ld_beta, int beta_col0, float* A, float* B, int* dev_err, void* stream);

/* inv = (I + sym(A))^-1 by Gauss-Jordan without pivoting (the pivots are ratios of leading
 * minors); info[f, h] = order of the first non-positive leading minor (0 = SPD).
 * text_frame >= 0: s0 = text_scale * B inv of it.  inv_split (head_dim 128, optional): the
 * inverses again as bf16 hi halves [F, H, 128, 128] followed by the lo halves
 * (hi = bf16(x), lo = bf16(x - hi)), the operands of vdn_bidir_scan_tc.
 * Replaces: branch.py:148-160 (VdnDelta.factor_apply), :62-71 (cholesky_ex info),
 *           :649-670 (_text_state). */
int vdn_delta_factor(const float* A, const float* B, int F, int H, int D, float* inv, int* info,
                     int text_frame, float text_scale, float* s0, void* inv_split, void* stream);

/* The sana_scaled factor: M = I - inv_tokens * A per frame, row-major into M (optional) and,
 * for head_dim 128, transposed as bf16 hi / lo halves into M_split (optional; the operand of
 * vdn_bidir_scan_tc).  text_frame >= 0: s0 = text_scale * (text_inj_scale * B[text_frame]).
 * Replaces: branch.py:163-177 (SanaDelta.factor_apply), :649-670 (_text_state). */
int vdn_sana_factor(const float* A, const float* B, int F, int H, int D, float inv_tokens, float* M, void* M_split,
                    int text_frame, float text_inj_scale, float text_scale, float* s0, void* stream);

/* inj_scale = 0 (vdn_solve): prefix_t = (B_t + prefix_{t-1} diag(alpha_t)) inv_t (t up),
 * suffix likewise (t down), both from s0 (NULL = zero).  inj_scale > 0 (sana_scaled, inv = M):
 * prefix_t = prefix_{t-1} diag(alpha_t) M_t + inj_scale B_t.  Replaces: branch.py:297-333
 * (run_scans_*), runtime.py:118-150 (_run_scans_shared). */
int vdn_bidir_scan(const float* inv, const float* B, const float* alpha, const float* s0, int F, int H, int D,
                   float inj_scale, float* prefix, float* suffix, void* stream);

/* The same scan on tensor cores (head_dim 128): one CTA per (head, direction) keeps the state
 * in TMEM and multiplies by the inverse in three bf16 passes (hi*hi + hi*lo + lo*hi, fp32
 * accumulation).  inv_split from vdn_delta_factor over F_inv >= F frames; B [F_inv, H, 128, 128].
 * Replaces: branch.py:297-333 (run_scans_*). */
int vdn_bidir_scan_tc(const void* inv_split, const float* B, const float* alpha, const float* s0, int F,
                      int F_inv, int H, float inj_scale, float* prefix, float* suffix, int* dev_err, void* stream);

/* Gather with alpha bridge, readout Q S^T, RMSNorm over D, x output gate, into
 * out[out_row0 + f*T + s, h*D + v] for the F frames f0 .. f0+F-1 of a clip of F_all frames
 * (Q [F, H, T, D] and gate rows hold those frames; prefix, suffix, alpha, lo, hi cover the
 * clip; f0 = 0, F_all = F for a whole clip).  Replaces: branch.py:345-396
 * (gather_linear_state), branch.py:780, :494-530 (readout, linear_epilogue), and with f0 > 0
 * the per-tile readout of runtime.py:516-543 (_projected_delta_tiled). */
int vdn_readout(const void* Q, int F, int H, int T, int D, const float* prefix, const float* suffix,
                const float* alpha, const float* s0, const int* lo, const int* hi, int use_alpha,
                const float* norm_w, const void* gate, long long ld_gate, void* out, long long ld_out,
                long long out_row0, int f0, int F_all, void* stream);

/* Tensor-core readout for head_dim 128: gather + alpha bridge into a bf16 state, R = Q S^T and
 * the output-gate up-projection G = og_down og_up^T as tcgen05 MMAs, then RMSNorm(D) x norm_w x
 * sigmoid(G + og_bias) into out[out_row0 + f*T + s, h*128 + v].  og_down [F*T, 128] bf16,
 * og_up [H*128, 128] bf16.  Frames f0 .. f0+F-1 of a clip of F_all, as in vdn_readout.
 * out, prefix, suffix, s0, norm_w and og_bias must be 16-byte aligned (kMisaligned otherwise).
 * Replaces: branch.py:345-396, :494-530, :754-758, :780. */
int vdn_readout_tc(const void* Q, int F, int H, int T, const float* prefix, const float* suffix,
                   const float* alpha, const float* s0, const int* lo, const int* hi, int use_alpha,
                   const float* norm_w, const void* og_down, const void* og_up, const float* og_bias,
                   void* out, long long ld_out, long long out_row0, int f0, int F_all, int* dev_err,
                   void* stream);

/* fp32 column block -> bf16 (output-gate bottleneck rounding, branch.py:755). */
int vdn_cast_rows(const float* in, long long ld_in, int col0, int rows, int cols, void* out, long long ld_out,
                  void* stream);

/* Rotary position embedding, split-half pairing, in place on `slots` consecutive heads of D
 * bf16 features per row (the normalised q heads then k heads): for j < rot/2 the pair
 * (x[j], x[j + rot/2]) becomes f[row, j] (x[j], x[j + rot/2])^T, f fp32 [rows, rot/2, 2, 2]
 * (ComfyUI's freqs layout [[cos, -sin], [sin, cos]]) with row stride ld_freqs (0: shared by
 * every row); features >= rot unchanged.  rot even, rot <= D.
 * Replaces: the RoPE half of ck.rms_rope_split_half_ (hybrid.py:271-292). */
int vdn_rope_split_half(void* qk, long long ld, int rows, int slots, int D, int rot, const float* freqs,
                        long long ld_freqs, void* stream);

/* ---------------------------------------------------------------- DiT block -------- */

/* Per-row int8 of bf16 rows whose max |x| per row is already in amax [rows] (e.g. from
 * vdn_gemm_block's row_amax): same codes and scales as vdn_quant_int8_rows, one streaming pass.
 * K % 8 == 0; 16-byte aligned x rows, 8-byte aligned q rows. */
int vdn_quant_int8_rows_amax(const void* x, long long ldx, int rows, int K, const float* amax, void* q,
                             long long ldq, float* scale, void* stream);

/* out / q[r] = RMSNorm(x[r]) * norm_w * (1 + scale_tab[g]) + shift_tab[g], g = row_group[r].
 * x [rows, ldx] bf16, norm_w [hidden] fp32, tables [groups, ld_tab] bf16 (NULL: 0),
 * row_group [rows] int32 (NULL: group 0).  Writes out [rows, ldo] bf16 and/or per-token int8
 * q [rows, ldq] with q_scale [rows] fp32.  hidden % 8 == 0.
 * Replaces: block_kernels.py:85-89 (_pre_body) and the activation quantiser of the INT8 MLP. */
int vdn_adaln_rmsnorm(const void* x, long long ldx, int rows, int hidden, const float* norm_w, float eps,
                      const void* scale_tab, const void* shift_tab, long long ld_tab, const int* row_group,
                      void* out, long long ldo, void* q, long long ldq, float* q_scale, void* stream);

/* C [M, N'] bf16 = residual + gate[row_group[row]] * act(alpha * dev_scale0 * dev_scale1 * row_scale * col_scale
 * * (A B^T) + col_bias).  act: 0 none, 2 GELU (erf), 3 SwiGLU (B's rows interleaved in 128-row
 * gate / up blocks, N % 256 == 0, N' = N / 2).  A: one source, K-concatenated (A2 for
 * k >= k_split) or grouped-K (kg > 0, K / kg slabs group_stride apart).  residual [M, ld_res]
 * bf16 and (row_group [M] int32, group_gate [groups, ld_gate] bf16) are optional; row_amax [M] fp32
 * (optional, zeroed by the caller) receives each row's max |C| for vdn_quant_int8_rows_amax.
 * Replaces: block_kernels.py:92-93 (_post_body) fused into the projection that feeds it,
 * :113-146 (fc1, SwiGLU, fc2). */
int vdn_gemm_block(int kind, const void* A, long long lda, const void* A2, long long lda2, long long k_split,
                   long long group_stride, int kg, const void* B, long long ldb, void* C, long long ldc, int M,
                   int N, int K, float alpha, const float* dev_scale0, const float* dev_scale1,
                   const float* row_scale, const float* col_scale, const float* col_bias, int act,
                   const void* residual, long long ld_res, const int* row_group, const void* group_gate,
                   long long ld_gate, float* row_amax, int* dev_err, void* stream);

/* ---------------------------------------------------------------- diagnostics ----- */

/* Number of kernels this library has launched since it was loaded (host-side count, one per
 * launch; a caller takes the difference around a region to count its launches). */
long long vdn_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* VDN_B200_H */
