/*
 * oumu_attn.h — C ABI of the B200 (sm_100a) attention hot path for oumu / VoxCPM2.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream, launches asynchronously on that
 * stream, and returns an oumu_status. Nothing here allocates device memory, synchronises the stream or reads
 * device memory from the host, so every call can be recorded inside a CUDA graph capture (positions and lengths
 * are read on the device, grids depend only on the shape arguments). The caller owns every buffer.
 *
 * Layouts are the reference engine's (hayatree/oumu):
 *   qkv    bf16 [rows][(nq + 2*nk) * hd]     q heads, then k heads, then v heads      (src/model.rs:18)
 *   cache  bf16 [slots][nk][maxlen][hd]      one K and one V cache per layer          (src/model.rs:130-133)
 *   att    bf16 [rows][nq * hd]              attention output, input of o_proj        (src/model.rs:624)
 *   cos/sin fp32 [maxlen][hd / 2]            bf16-rounded rotary tables               (src/model.rs:337-349)
 *
 * bf16 buffers are passed as void* (raw 16-bit storage, like the reference's u64 device pointers).
 */
#ifndef OUMU_ATTN_H
#define OUMU_ATTN_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *oumu_stream_t; /* the same handle as cudaStream_t / CUstream */

typedef enum {
    OUMU_OK = 0,
    OUMU_ERR_INVALID = 1,     /* an argument is out of range (null pointer, negative size, nq % nk != 0 ...) */
    OUMU_ERR_UNSUPPORTED = 2, /* a valid shape these kernels do not implement (hd not 64/128, group > 8) */
    OUMU_ERR_WORKSPACE = 3,   /* the workspace passed is smaller than the *_workspace() query asked for */
    OUMU_ERR_CUDA = 4,        /* a CUDA runtime/driver call failed (launch, tensor-map encode, ...) */
    OUMU_ERR_DEVICE = 5       /* a kernel recorded an error on the device (see oumu_device_error) */
} oumu_status;

/* Human-readable name of a status code. */
const char *oumu_status_string(int status);

/* Last CUDA error string seen by this library on the calling thread ("" if none). */
const char *oumu_last_cuda_error(void);

/*
 * Programmatic dependent launch, process-wide, off by default; returns the previous setting. Applies to the decode
 * kernels (oumu_decode_prologue, oumu_attn_decode, oumu_attn_decode_step), oumu_gemm, the glue kernels
 * oumu_rmsnorm, oumu_silu_mul and oumu_pointwise (include/oumu_step.h), and the tensor-memory attention kernels of
 * oumu_attn_full, oumu_attn_full_rope and oumu_attn_prefill_kv (causal prefill, short sequences). When on, these
 * kernels are launched so that they may start while the preceding kernel in the stream is still running: their
 * set-up and their reads of constant data (GEMM weights, norm weights, cache positions below each take's newest
 * position) overlap the preceding kernel; everything it may write (q, activations, the newest position) is read,
 * and every global write made, only after it has completed. Most let their successor start at once; the attention
 * kernels that hold all of an SM's tensor memory take it only after the preceding kernel has completed and let
 * their successor in only once they hold it. The caller guarantees that the preceding kernels
 * of the same step do not write `pos`/`lens`, cache positions below the newest one, or weights (true of the
 * reference's step, where ctr advances only in step_end, src/model.rs:771, and kv_write writes only position *pos,
 * src/model.rs:590-595). Captured into CUDA graphs as programmatic edges.
 */
int oumu_set_pdl(int enable);

/*
 * Rotary tables, host side. Replaces rotary_tables (src/model.rs:337-349): for position p < maxlen and
 * i < hd/2, fr = (p * (1 / ext[i])) * (1 / 10000^(2i/hd)) in fp32, cos/sin rounded to bf16 and stored as fp32.
 * ext == NULL means ext[i] = 1 (plain base-10000 RoPE). cos_out/sin_out are HOST arrays of maxlen*hd/2 floats.
 */
int oumu_rotary_tables(int maxlen, int hd, const double *ext, float *cos_out, float *sin_out);

/*
 * In-place rotary embedding on the q and k heads of a fused qkv buffer.
 * Replaces the `rope` kernel (kernels/voxcpm.cu:100-115), launched at src/model.rs:544-550 (prefill/DiT/LocEnc,
 * seq > 0: row r uses position r % seq) and src/model.rs:581-587 (decode, seq == 0: every row uses *pos).
 * Bit-exact with the reference: x1' = bf16(x1*c - x2*s), x2' = bf16(x2*c + x1*s) in fp32.
 */
int oumu_rope(void *qkv, const float *cos_t, const float *sin_t, const int *pos, int rows, int seq, int nq,
              int nk, int hd, oumu_stream_t stream);

/*
 * Copy k and v of `rows` consecutive positions of every slot into the per-layer caches, starting at *pos
 * (or 0 when pos == NULL). qkv rows are [slot * rows + i]. Bit-exact copy.
 * Replaces `kv_write` (kernels/voxcpm.cu:117-129) launched with grid (rows, slots, nk) at src/model.rs:553-559
 * (prefill: slots = 1, pos = NULL) and src/model.rs:590-595 (decode: rows = 1, slots = B, pos = ctr).
 */
int oumu_kv_write(const void *qkv, void *kc, void *vc, const int *pos, int slots, int rows, int nq, int nk, int hd,
                  int maxlen, oumu_stream_t stream);

/*
 * Decode prologue, one launch per layer: for every take s at position p_s, rotate its q and k heads in place
 * (skipped when cos_t == NULL, e.g. the residual LM, src/model.rs:445) and write its k and v into cache slot s
 * at p_s. p_s = lens[s] - 1 when lens != NULL (per-take lengths), else *pos for every take.
 * Replaces the rope + kv_write pair of Engine::step_tf (src/model.rs:580-595); same arithmetic as oumu_rope.
 */
int oumu_decode_prologue(void *qkv, void *kc, void *vc, const float *cos_t, const float *sin_t, const int *pos,
                         const int *lens, int B, int nq, int nk, int hd, int maxlen, oumu_stream_t stream);

/*
 * Bytes of device workspace oumu_attn_decode needs for this shape (partials of the split-KV pass plus one
 * counter per (take, kv head)). The counters must be zero before the first call: allocate the workspace
 * zero-filled (as src/gpu.rs:108-113 does) or call oumu_attn_decode_reset once. Every call leaves them zero.
 */
size_t oumu_attn_decode_workspace(int B, int nq, int nk, int hd, int maxlen);

/* Zero the combine counters of a decode workspace (asynchronous memset on `stream`). */
int oumu_attn_decode_reset(void *workspace, size_t workspace_bytes, int B, int nq, int nk, int hd, int maxlen,
                           oumu_stream_t stream);

/*
 * Split-KV GQA decode attention with the cross-split combine fused in (one launch).
 * For take s, q head h (kv head h / (nq/nk)): out[s][h*hd + d] = bf16( sum_j e^(q.k_j*scale - m) v_j[d] / sum_j
 * e^(q.k_j*scale - m) ) over positions j < L_s, with L_s = lens[s] (lens != NULL) or *pos + 1 (the reference's
 * shared position). q is read from qkv row s (already rotated), k/v from cache slot s.
 * Replaces attn_decode + attn_combine (kernels/voxcpm.cu:131-185), launched at src/model.rs:596-615; `out` is
 * the reference's sc.att [B][nq*hd], `workspace` takes the place of StepBufs::att_part (src/model.rs:237).
 * The workspace the reference allocates for att_part is always enough: with less than
 * oumu_attn_decode_workspace() bytes the kernel uses fewer CTAs, down to a minimum it checks.
 * Supported: hd in {64, 128}, nq / nk in 1..8, B <= 4096 (B <= 1203 for hd 128: the per-take length table shares
 * the kernel's shared memory with the KV stages), B * nk * maxlen < 2^31; other shapes OUMU_ERR_UNSUPPORTED.
 */
int oumu_attn_decode(const void *qkv, const void *kc, const void *vc, void *out, void *workspace,
                     size_t workspace_bytes, const int *pos, const int *lens, int B, int nq, int nk, int hd,
                     int maxlen, float scale, oumu_stream_t stream);

/*
 * Decode attention that allocates nothing and takes no workspace: oumu_attn_decode with its scratch (split-KV
 * partials and combine counters) in a static device array of OUMU_DECODE_STATIC_SCRATCH_BYTES that the library
 * holds on every device that loads it, until the process exits. For callers that cannot give the library device
 * memory: a plug-in that receives only its input and output buffers from an engine that owns every device
 * allocation, or a host whose memory policy forbids a library to allocate on its own. No counterpart in the
 * reference (its att_part is allocated by the engine, src/model.rs:237).
 * Limits, checked before anything is queued (a rejected call leaves the stream and the array untouched):
 *   - every limit of oumu_attn_decode: hd in {64, 128}, nq / nk in 1..8, B <= 4096, B * nk * maxlen < 2^31, and
 *     the per-take length table in shared memory, which caps B at 1203 for hd 128 (OUMU_ERR_UNSUPPORTED);
 *   - the array holds one counter per (take, kv head) plus at least one CTA's partials: B * nk <= 522,176 for
 *     hd 128 and <= 523,200 for hd 64, else OUMU_ERR_WORKSPACE with a message in oumu_last_cuda_error. Below one
 *     CTA per SM's worth of room the kernel runs on fewer CTAs.
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress) with that device
 * current, in its primary context, and keeps it: make that first call before any stream capture, and do not reset
 * the device afterwards. Every call clears the counters (an asynchronous memset on `stream`) and then uses the
 * shared array, so calls that can overlap on the GPU (other streams, other host threads) race with each other:
 * serialise them.
 */
#define OUMU_DECODE_STATIC_SCRATCH_BYTES (2 * 1024 * 1024)
int oumu_attn_decode_static(const void *qkv, const void *kc, const void *vc, void *out, const int *pos,
                            const int *lens, int B, int nq, int nk, int hd, int maxlen, float scale,
                            oumu_stream_t stream);

/*
 * One decode layer in one launch: the decode prologue and the decode attention of oumu_decode_prologue +
 * oumu_attn_decode fused. For every take s at position p_s (lens[s] - 1, or *pos): its k at p_s is rotated
 * (cos_t/sin_t; NULL for no rope) and written with v into cache slot s, its q is rotated in registers, and the
 * attention over positions <= p_s is written to `out`, bit-identical to the two separate calls. Buffer effects
 * differ only in qkv: the rotated k is written back into qkv as rope does, the q heads are left unrotated (the
 * reference reads qkv no further after attention, src/model.rs:622-632).
 * Replaces the rope + kv_write + attn_decode + attn_combine sequence of Engine::step_tf (src/model.rs:580-615).
 * Same workspace as oumu_attn_decode.
 */
int oumu_attn_decode_step(void *qkv, void *kc, void *vc, void *out, void *workspace, size_t workspace_bytes,
                          const float *cos_t, const float *sin_t, const int *pos, const int *lens, int B, int nq,
                          int nk, int hd, int maxlen, float scale, oumu_stream_t stream);

/*
 * Attention inside independent sequences of length `seq` held in a fused qkv buffer of `rows` = nseq * seq rows;
 * causal masks future keys. out[r][h*hd + d] = bf16( sum_j p_j v_j[d] / sum_j p_j ), p_j = e^(q_r.k_j*scale - m).
 * Replaces attn_full (kernels/voxcpm.cu:262-297), launched at src/model.rs:561-567 for the causal prefill
 * (seq = T), the local encoder (seq = 5) and the LocDiT (seq = 11, all takes x 2 CFG branches in one call).
 * seq <= 16 runs the fused small-sequence kernel (one warp per (sequence, q head), tensor-core mma);
 * longer sequences run the tcgen05/TMEM flash-attention kernel fed by TMA.
 * Supported: hd in {64, 128}; nq % nk == 0.
 */
int oumu_attn_full(const void *qkv, void *out, int rows, int seq, int causal, int nq, int nk, int hd, float scale,
                   oumu_stream_t stream);

/*
 * Rope + attention of one layer of Engine::full in one launch, for the small sequences of the DiT and the local
 * encoder: out = oumu_attn_full of qkv with q and k rotated at positions r % seq (the tables of oumu_rope, at least
 * seq rows), bit-identical to oumu_rope followed by oumu_attn_full. qkv itself is not modified.
 * Replaces the rope + attn_full launches of src/model.rs:541-567 (kernels/voxcpm.cu:100-115, 262-297).
 * Supported: seq <= 16, nq / nk >= 2, (nq / nk) * seq <= 128, hd in {64, 128}; other shapes OUMU_ERR_UNSUPPORTED.
 */
int oumu_attn_full_rope(const void *qkv, void *out, const float *cos_t, const float *sin_t, int rows, int seq,
                        int causal, int nq, int nk, int hd, float scale, oumu_stream_t stream);

/*
 * Replicate slot 0 of a per-layer cache [B][nk][maxlen][hd] into slots 1..B-1 for positions < T.
 * Replaces kv_replicate (kernels/voxcpm.cu:407-413), launched per K and V cache at src/model.rs:705-717.
 * Bit-exact copy; reads slot 0 once and writes the other B-1 slots.
 */
int oumu_kv_replicate(void *cache, int B, int nk, int maxlen, int hd, int T, oumu_stream_t stream);

/*
 * Causal prefill of one prompt with the KV epilogue, one launch: out = the causal attention of qkv's T rows (as
 * oumu_attn_full(qkv, out, T, T, 1, ...)), and the prompt's k and v (already rotated) written into positions [0, T) of
 * every one of the `slots` take slots of kc and vc ([slots][nk][maxlen][hd]); positions >= T are not touched.
 * Replaces, per layer, kv_write into slot 0 + attn_full (src/model.rs:553-567) and the later kv_replicate into slots
 * 1..B-1 (src/model.rs:705-717). T > 16 (the tensor-core path), T <= maxlen; caches bit-exact.
 */
int oumu_attn_prefill_kv(const void *qkv, void *out, void *kc, void *vc, int T, int slots, int nq, int nk, int hd,
                         int maxlen, float scale, oumu_stream_t stream);

/*
 * Device-side error word of this library on the current device: 0 when no kernel recorded an error (a bounded
 * wait that ran out, a length outside [1, maxlen]). Synchronises the device. reset != 0 clears it.
 */
int oumu_device_error(int reset);

/*
 * Failure detection. No reference counterpart: the reference's kernels have no waits and report nothing
 * (src/gpu.rs:11 only propagates launch errors).
 *
 * oumu_set_wait_limit_ns: the time after which a bounded device-side wait of this library's kernels (a pipeline
 * stage that never fills, a hand-off that never comes) gives up: the kernel records OUMU_DEVERR_TIMEOUT in the
 * device error word, stops waiting for anything, lets every copy it issued land and exits; its outputs are then
 * unspecified, the decode workspace's counters are left at zero, and the context stays usable. Default 2 s; ns = 0
 * restores it. Applies to the current device, to launches made after the call (a synchronous copy to the device:
 * not inside a stream capture).
 *
 * oumu_test_drop_last_tile: fault injection for tests of that path, process-wide, off (0) by default; returns the
 * previous setting. While on, every decode launch (oumu_attn_decode, oumu_attn_decode_static,
 * oumu_attn_decode_step) leaves the last 32-position tile of its first CTA's range unloaded, so the consumer that
 * owns it waits until the limit. Nothing faults, traps or hangs: the wait is bounded.
 */
int oumu_set_wait_limit_ns(unsigned long long ns);
int oumu_test_drop_last_tile(int on);

#ifdef __cplusplus
}
#endif

#endif /* OUMU_ATTN_H */
