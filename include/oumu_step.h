/*
 * oumu_step.h — C ABI of the per-step kernels around the attention in oumu's decoding step (VoxCPM2 on sm_100a).
 *
 * These replace the reference's glue kernels between the GEMMs of Engine::full / Engine::step_tf / Engine::step
 * (src/model.rs:532-773, kernels in kernels/voxcpm.cu). Same conventions as oumu_attn.h: plain device pointers,
 * bf16 buffers as void*, asynchronous on `stream`, an oumu_status return, nothing allocated and nothing read back,
 * so every call can be recorded in a CUDA graph. Row widths must be multiples of 8 and buffers 16-byte aligned
 * (the kernels move 16-byte vectors).
 */
#ifndef OUMU_STEP_H
#define OUMU_STEP_H

#include "oumu_attn.h"

#ifdef __cplusplus
extern "C" {
#endif

/*
 * RMS norm of `rows` rows of `dim` elements (dim 1024 or 2048): out = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w).
 * With d != NULL the residual is updated first, res = bf16(res + d), and the norm is of the updated row.
 * Replaces rmsnorm (kernels/voxcpm.cu:43-52, launched src/model.rs:539) and add_rmsnorm (kernels/voxcpm.cu:55-67,
 * launched src/model.rs:625,629).
 */
int oumu_rmsnorm(void *res, const void *d, const void *w, void *out, int rows, int dim, float eps,
                 oumu_stream_t stream);

/*
 * SwiGLU product: gu = [gate | up] per row (2F wide), out[r][c] = bf16(bf16(silu(gate)) * up), out [rows][F].
 * Replaces silu_mul (kernels/voxcpm.cu:92-99, launched src/model.rs:627).
 */
int oumu_silu_mul(const void *gu, void *out, int rows, int F, oumu_stream_t stream);

/*
 * In place over n elements (n % 8 == 0). op 0: silu (silu_inplace, kernels/voxcpm.cu:80-83, src/model.rs:755).
 * op 1: FSQ, h = bf16(rint(bf16(bf16(tanh(h)) * scale)) / scale) (fsq_act, kernels/voxcpm.cu:370-375,
 * src/model.rs:760).
 */
int oumu_pointwise(void *x, long n, int op, float scale, oumu_stream_t stream);

/*
 * DiT input sequences (seq == 11): for 2B rows, [mu0, mu1, t, cond x4, x x4] x H; rows < B take mu [B][2][H],
 * rows >= B zeros; condp and xp [B][4][H]; temb one row of H. Replaces dit_build (kernels/voxcpm.cu:299-315,
 * src/model.rs:737-743); `rows` must be 2B.
 * Local-encoder sequences (seq == 5): for `rows` patches, [special, x0..x3] x H with temb = the special token and
 * mu, condp unused (may be NULL). Replaces enc_build (kernels/voxcpm.cu:325-331, src/model.rs:637).
 */
int oumu_build_seq(void *seq_out, const void *mu, const void *temb, const void *condp, const void *xp, int rows,
                   int B, int seq, int H, oumu_stream_t stream);

/*
 * Classifier-free guidance (CFG-Zero*) and one Euler step of the DiT for B takes: x [B][256] -= dt * guided
 * velocity, reading frame t of DiT output row r (rows 0..B-1 conditional, B..2B-1 unconditional) at
 * out[(r * seq + first + t) * 64 + c]. seq = 4, first = 0 is the reference's gathered layout; seq = 11, first = 7
 * reads the DiT's full output without gathering. Replaces cfg_euler (kernels/voxcpm.cu:334-345, src/model.rs:748)
 * and, with seq = 11, gather_rows (kernels/voxcpm.cu:317-323, src/model.rs:745).
 */
int oumu_cfg_euler(void *x, const void *out, int B, int seq, int first, float dt, float cfg, oumu_stream_t stream);

/*
 * End of a decoding step, one block: patch [B][256] -> patches[s][ctr[1]] (if ctr[1] < max_steps); stop[s] = ctr[1]
 * for a take whose stop logits [B][2] ask to stop (logit 1 > logit 0) after more than min_len patches and that has
 * not stopped; then ctr[0] += 1, ctr[1] += 1 and, when lens != NULL, lens[s] += 1 for every take.
 * Replaces step_end (kernels/voxcpm.cu:415-433, src/model.rs:766-772); `lens` is this library's per-take variant.
 */
int oumu_step_end(const void *stop_logits, const void *patch, void *patches, int *stop, int *ctr, int *lens, int B,
                  int min_len, int max_steps, oumu_stream_t stream);

/*
 * The decoding loop as one graph launch, with the stop test on the device: Engine::decode (src/model.rs:777-796)
 * replays the step graph and reads `stop` back after every step; this runs
 *     while (ctr[1] < max_steps && some stop[s] < 0 for s < B) { step; }
 * as a CUDA WHILE conditional node around a copy of `step_graph` (a cudaGraph_t, e.g. torch's
 * CUDAGraph(keep_graph=True).raw_cuda_graph(); it may hold kernel, memset, memcpy and child-graph nodes only),
 * so the host reads `stop` once, after the loop. `stop` [B], `ctr` [4] (ctr[1] = patches so far, advanced by the
 * step's oumu_step_end) and `status` [2] are device int buffers the step graph and the loop share; after a launch
 * status[0] = steps run and status[1] = 1 if the loop ended at max_steps steps while ctr[1] had not reached
 * max_steps (a step graph that does not advance ctr[1]), else 0. The loop holds its own copy of the step graph:
 * `step_graph` may be destroyed after create. One loop per step graph may exist at a time (a CUDA rule for graphs
 * with conditional nodes).
 */
typedef struct oumu_decode_loop_s *oumu_decode_loop_t;
int oumu_decode_loop_create(void *step_graph, const int *stop, const int *ctr, int *status, int B, int max_steps,
                            oumu_decode_loop_t *loop);
int oumu_decode_loop_launch(oumu_decode_loop_t loop, oumu_stream_t stream);
int oumu_decode_loop_destroy(oumu_decode_loop_t loop);

/*
 * y[m][n] (row pitch ldy) = bf16(sum_k x[m][k] * W[n][k] (+ bias[n])) for m < M, n < N: x bf16 [M][K] with row
 * pitch ldx (>= K, a multiple of 8), W bf16 [N][K] contiguous, bias bf16 [N] or NULL, fp32 accumulation, one
 * rounding after the bias. K must be a multiple of 64; x and W 16-byte aligned. Replaces Lin::fwd -> Gpu::gemm
 * (src/model.rs:27-45, src/gpu.rs:186-229: gemv_* for M <= 8, cuBLAS gemm_ex above; fill_bias + beta = 1,
 * kernels/voxcpm.cu:70-76). One launch of thread-block clusters, no workspace, deterministic; with oumu_set_pdl(1)
 * it may start during the preceding kernel and stream its first weights before waiting for it.
 */
int oumu_gemm(const void *x, int ldx, const void *w, void *y, int ldy, const void *bias, int M, int N, int K,
              oumu_stream_t stream);

/*
 * The SwiGLU MLP's input projection and activation in one launch: act[m][i] (row pitch ldact >= F) =
 * bf16(bf16(silu(g)) * u) for i < F, with g = bf16(x[m] . Wg[i] (+ bg[i])) and u = bf16(x[m] . Wu[i] (+ bu[i])), the
 * values oumu_gemm would store for the gate | up projection and the arithmetic of silu_mul (kernels/voxcpm.cu:92-99):
 * the output is bit-identical to oumu_gemm into [M][2F] followed by oumu_silu_mul, without the [M][2F] intermediate
 * or the second launch (Engine's Mlp: the gate|up Lin, then silu_mul, src/model.rs:627-628). w_il is the gate|up
 * weight [2F][K] with its rows interleaved in groups of 8: rows [16j, 16j + 8) are gate rows [8j, 8j + 8) and rows
 * [16j + 8, 16j + 16) are up rows [8j, 8j + 8) (bias_il, if not NULL, interleaved the same way); a host permutes the
 * weight once when it loads it. F a multiple of 8; the other requirements are oumu_gemm's with N = 2F.
 */
int oumu_gemm_swiglu(const void *x, int ldx, const void *w_il, void *act, int ldact, const void *bias_il, int M,
                     int F, int K, oumu_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* OUMU_STEP_H */
