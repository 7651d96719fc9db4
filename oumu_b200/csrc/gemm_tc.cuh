// Weight-streaming GEMM on the 5th-generation tensor cores for the projections of the decoding step:
// y[M][N] = bf16(x[M][K] . W[N][K]^T (+ bias[N])), fp32 accumulation, the bias added before the single rounding
// (the reference's Lin::fwd -> Gpu::gemm, src/model.rs:27-45, src/gpu.rs:186-229, kernels/voxcpm.cu:70-76).
//
// At decode sizes (M = takes per GPU, 32-64) the cost is reading W once:
//   * W is the MMA's A operand (M = 128 weight rows per tile) and the tokens its N (TN = 32/64/128 per tile):
//     D^T[128 x TN] accumulates in TMEM. One tcgen05.mma occupies the SM's tensor pipe for ~160 cycles whatever
//     its N, so an SM consumes 4 KB of W per instruction (~50 GB/s); the kernel therefore spreads every GEMM over
//     (nearly) all SMs.
//   * Each output tile (TN tokens x 128 weight rows) belongs to one thread-block cluster of C CTAs (C <= 8), which
//     split its K range evenly; the host picks the largest C whose grid is resident in one wave (occupancy query).
//     The C partial accumulators meet in distributed shared memory: CTA c owns rows [c*R, (c+1)*R) of the tile,
//     every CTA pushes those rows of its partial into CTA c's inbox (st.shared::cluster), and after one cluster
//     barrier each CTA sums its rows over the C partials in rank order (deterministic), adds the bias and writes y.
//     No global atomics, no partials in HBM, nothing read remotely after the barrier.
//   * Warp roles: warp 0 issues TMA (the weight boxes of the first stages before griddepcontrol.wait: weights do
//     not depend on the preceding kernel, so their loads overlap its tail), warp 1 owns TMEM and issues
//     tcgen05.mma, warps 2-5 move the accumulator from TMEM to the owners' inboxes (thread = weight row); all six
//     warps reduce.
// SwiGLU form (Params::act): W holds the gate and up rows of an MLP interleaved in groups of 8 (rows [16j, 16j + 8)
// are gate rows [8j, 8j + 8), rows [16j + 8, 16j + 16) the up rows of the same indices), so each owner's row range
// (whole groups of 16) holds both halves of its outputs; the reduction rounds gate and up to bf16 as the plain form
// would store them and writes act[m][8j + i] = bf16(bf16(silu(gate)) * up), the arithmetic of the separate
// silu_mul kernel (kernels/voxcpm.cu:92-99), so the result is bit-identical to the GEMM followed by silu_mul.
// All mbarrier waits are bounded (mbar_wait); on a timeout the kernel records the error and still reaches the
// cluster barrier (its output is then garbage, and the error word says so).
#pragma once
#include "common.cuh"

namespace gm {

constexpr int BW = 128;               // weight rows per tile (MMA M)
constexpr int BK = 64;                // K per stage: one 128-byte swizzled row of bf16
constexpr int NTHREADS = 6 * 32;      // TMA, MMA, 4 epilogue warps
constexpr int W_BYTES = BW * BK * 2;  // 16 KB
constexpr int MAX_SPLIT = 8;          // portable cluster size

// Rows of a tile each CTA of a split-C cluster owns: whole groups of 8, or of 16 in the SwiGLU form (a gate group
// and its up group).
__host__ __device__ constexpr int rows_per_owner(int split, int act = 0) {
    return ((BW / split + (BW % split ? 1 : 0) + (act ? 15 : 7)) / (act ? 16 : 8)) * (act ? 16 : 8);
}

template <int TN, int STAGES>
struct Cfg {
    static_assert(TN % 32 == 0 && TN >= 32 && TN <= 128, "token tile");
    static constexpr int X_BYTES = TN * BK * 2;
    static constexpr int STAGE_BYTES = W_BYTES + X_BYTES;  // a multiple of 1024: every box starts 1024-aligned
    static constexpr int BAR_BYTES = 1024;                 // barriers first, so the stages stay 1024-aligned
    static constexpr int STAGE_OFF = BAR_BYTES;
    static constexpr int INBOX_OFF = STAGE_OFF + STAGES * STAGE_BYTES;
    static constexpr uint32_t TMEM_COLS = TN;              // 32, 64 or 128: a power of two >= 32
    // inbox: the split partials of the owned rows, [split][rows_per_owner][TN] fp32
    static constexpr int inbox_bytes(int split, int act = 0) { return split * rows_per_owner(split, act) * TN * 4; }
    static constexpr int smem_bytes(int split, int act = 0) {  // + alignment
        return INBOX_OFF + inbox_bytes(split, act) + 1024;
    }
};

struct Params {
    bf16 *y;
    const bf16 *bias;
    int ldy, M, N;
    int NT, KB;  // weight tiles, K blocks of 64
    int split;   // CTAs per tile = the cluster size
    int act;     // 0: y = x.W^T (+ bias); 1: the SwiGLU form (N = 2F interleaved rows, y [M][F])
};

// One item of the SwiGLU reduction: token t0 + tok, interleaved rows [n, n + 16) of W (8 gate rows, then the 8 up
// rows of the same outputs), summed over the split partials in rank order; act outputs [n / 2, n / 2 + 8).
template <int TN>
__device__ __forceinline__ void swiglu_item(const Params &P, const float *inbox, int split, int rpo, int grp, int tok,
                                            int t0, int n, bool vec) {
    float v[16];
#pragma unroll
    for (int j = 0; j < 16; j++) v[j] = 0.f;
#pragma unroll
    for (int q = 0; q < MAX_SPLIT; q++) {  // rank order: the same sum on every run
        if (q < split) {
            const float *src = inbox + (q * rpo + grp * 16) * TN + tok;
#pragma unroll
            for (int j = 0; j < 16; j++) v[j] += src[j * TN];
        }
    }
    if (t0 + tok >= P.M || n + 16 > P.N) return;
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        // gate and up as the plain form stores them (bias added before the one rounding), then silu_mul's arithmetic
        const float g = bf2f(f2bf(P.bias ? v[j] + bf2f(P.bias[n + j]) : v[j]));
        const float u = bf2f(f2bf(P.bias ? v[8 + j] + bf2f(P.bias[n + 8 + j]) : v[8 + j]));
        o[j] = bf2f(f2bf(g / (1.f + __expf(-g)))) * u;
    }
    bf16 *yp = P.y + static_cast<long>(t0 + tok) * P.ldy + n / 2;
    if (vec) {
        uint4 w;
        w.x = pack_bf16x2(o[0], o[1]);
        w.y = pack_bf16x2(o[2], o[3]);
        w.z = pack_bf16x2(o[4], o[5]);
        w.w = pack_bf16x2(o[6], o[7]);
        *reinterpret_cast<uint4 *>(yp) = w;
    } else {
#pragma unroll
        for (int j = 0; j < 8; j++) yp[j] = f2bf(o[j]);
    }
}

template <int TN, int STAGES>
__global__ void __launch_bounds__(NTHREADS, 1)
    k_gemm(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx, const Params P) {
    using C = Cfg<TN, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    // the same 1024-aligned offset in every CTA of the cluster (the dynamic shared window starts at the same
    // offset in each), so an inbox address maps across the cluster
    const uint32_t raw_s = smem_u32(smem_raw);
    uint8_t *sm = smem_raw + ((1024u - (raw_s & 1023u)) & 1023u);
    const uint32_t sm_s = smem_u32(sm);
    const uint32_t stages = sm_s + C::STAGE_OFF;
    // barriers: FULL[s] (TMA -> MMA), EMPTY[s] (MMA -> TMA), AFULL (MMA -> epilogue); then the TMEM address slot
    auto full_b = [&](int s) { return sm_s + 8u * s; };
    auto empty_b = [&](int s) { return sm_s + 8u * (STAGES + s); };
    const uint32_t afull = sm_s + 8u * (2 * STAGES);
    const uint32_t tslot = sm_s + 8u * (2 * STAGES + 1);
    volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(sm + 8 * (2 * STAGES + 1));
    volatile int *abort_flag = reinterpret_cast<volatile int *>(sm + 8 * (2 * STAGES + 2));
    const float *inbox = reinterpret_cast<const float *>(sm + C::INBOX_OFF);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = P.split;
    const int rank = static_cast<int>(cluster_rank());
    const int tile = blockIdx.x / split;
    const int n0 = (tile % P.NT) * BW, t0 = (tile / P.NT) * TN;
    const int kb0 = rank * P.KB / split, kb1 = (rank + 1) * P.KB / split;
    const int n_units = kb1 - kb0;
    const int rpo = rows_per_owner(split, P.act);

    if (threadIdx.x == 0) {
        pdl_trigger();
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full_b(s), 1);
            mbar_init(empty_b(s), 1);
        }
        mbar_init(afull, 1);
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 1) {
        tmem_alloc(tslot, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // first half of a cluster barrier: the epilogue waits on it before its first store into a peer's inbox (a peer's
    // shared memory may be written only once that peer has started); the wait overlaps the main loop
    cluster_arrive_relaxed();

    if (warp == 0) {
        // ------------------------------ TMA producer ------------------------------
        if (lane == 0) {
            tma_prefetch_desc(&tw);
            tma_prefetch_desc(&tx);
            const int pre = n_units < STAGES ? n_units : STAGES;
            for (int i = 0; i < pre; i++) {  // weights first: independent of the preceding kernel
                mbar_expect_tx(full_b(i), C::STAGE_BYTES);
                tma_load_2d(stages + i * C::STAGE_BYTES, &tw, full_b(i), (kb0 + i) * BK, n0);
            }
            pdl_wait();
            for (int i = 0; i < pre; i++)
                tma_load_2d(stages + i * C::STAGE_BYTES + W_BYTES, &tx, full_b(i), (kb0 + i) * BK, t0);
            for (int i = pre; i < n_units; i++) {
                const int s = i % STAGES;
                if (!mbar_wait(empty_b(s), ((i / STAGES) - 1) & 1)) {
                    *abort_flag = 1;
                    break;
                }
                if (*abort_flag) break;
                mbar_expect_tx(full_b(s), C::STAGE_BYTES);
                tma_load_2d(stages + s * C::STAGE_BYTES, &tw, full_b(s), (kb0 + i) * BK, n0);
                tma_load_2d(stages + s * C::STAGE_BYTES + W_BYTES, &tx, full_b(s), (kb0 + i) * BK, t0);
            }
        }
        __syncwarp();
        cluster_wait();
    } else if (warp == 1) {
        // ------------------------------ MMA issuer ------------------------------
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16_f32(BW, TN, 0, 0);
            bool ok = true;
            for (int i = 0; i < n_units; i++) {
                const int s = i % STAGES;
                ok = mbar_wait(full_b(s), (i / STAGES) & 1);
                if (!ok) break;
                tc_fence_after();
                const uint32_t wb = stages + s * C::STAGE_BYTES, xb = wb + W_BYTES;
#pragma unroll
                for (int k = 0; k < BK / 16; k++)
                    tc_mma_ss(tmem, smem_desc_sw128(wb + k * 32, 16, 1024), smem_desc_sw128(xb + k * 32, 16, 1024),
                              idesc, (i == 0 && k == 0) ? 0u : 1u);
                tc_commit(empty_b(s));
            }
            tc_commit(afull);  // also on a timeout, so the epilogue does not wait in vain
            if (!ok) *abort_flag = 1;
        }
        __syncwarp();
        cluster_wait();
    } else {
        // ------------------------------ accumulator -> the owners' inboxes ------------------------------
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;  // weight row within the tile
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        const int owner = r / rpo;
        const uint32_t dst = cluster_map(sm_s + C::INBOX_OFF + ((rank * rpo + (r - owner * rpo)) * TN) * 4,
                                         static_cast<uint32_t>(owner));
        const bool ok = __all_sync(0xffffffffu, mbar_wait(afull, 0));
        cluster_wait();  // every CTA of the cluster has started: its inbox may be written
        if (ok) {
            tc_fence_after();
#pragma unroll 1
            for (int c0 = 0; c0 < TN; c0 += 32) {
                uint32_t acc[32];
                tmem_ld32(tmem + lane_off + c0, acc);
                tc_wait_ld();
#pragma unroll
                for (int c = 0; c < 32; c += 4)
                    st_cluster_f4(dst + (c0 + c) * 4, make_float4(__uint_as_float(acc[c]), __uint_as_float(acc[c + 1]),
                                                                  __uint_as_float(acc[c + 2]),
                                                                  __uint_as_float(acc[c + 3])));
            }
        } else {
            *abort_flag = 1;
        }
        tc_fence_before();
    }

    // ------------------------------ reduction of the owned rows ------------------------------
    cluster_sync();  // every partial has been pushed; nothing remote is touched after this
    pdl_wait();      // y is written only after the preceding kernel completed
    {
        const int r0 = rank * rpo, r1 = min(BW, r0 + rpo);
        const int gsz = P.act ? 16 : 8;  // rows per item
        const int groups = r1 > r0 ? (r1 - r0) / gsz : 0;
        const bool vec = (reinterpret_cast<uintptr_t>(P.y) & 15u) == 0 && (P.ldy & 7) == 0 &&
                         (reinterpret_cast<uintptr_t>(P.bias) & 15u) == 0;
        for (int item = threadIdx.x; item < TN * groups; item += NTHREADS) {
            const int grp = item / TN;
            const int tok = item - grp * TN;  // consecutive threads, consecutive tokens: no bank conflicts
            const int row = r0 + grp * gsz;
            if (P.act) {
                swiglu_item<TN>(P, inbox, split, rpo, grp, tok, t0, n0 + row, vec);
                continue;
            }
            float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int q = 0; q < MAX_SPLIT; q++) {  // rank order: the same sum on every run
                if (q < split) {
                    const float *src = inbox + (q * rpo + grp * 8) * TN + tok;
#pragma unroll
                    for (int j = 0; j < 8; j++) v[j] += src[j * TN];
                }
            }
            if (t0 + tok >= P.M) continue;
            const int n = n0 + row;
            bf16 *yp = P.y + static_cast<long>(t0 + tok) * P.ldy + n;
            if (vec && n + 8 <= P.N) {
                if (P.bias) {
                    const uint4 bu = *reinterpret_cast<const uint4 *>(P.bias + n);
                    const uint32_t bw[4] = {bu.x, bu.y, bu.z, bu.w};
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const float2 f = unpack_bf16x2(bw[j]);
                        v[2 * j] += f.x;
                        v[2 * j + 1] += f.y;
                    }
                }
                uint4 o;
                o.x = pack_bf16x2(v[0], v[1]);
                o.y = pack_bf16x2(v[2], v[3]);
                o.z = pack_bf16x2(v[4], v[5]);
                o.w = pack_bf16x2(v[6], v[7]);
                *reinterpret_cast<uint4 *>(yp) = o;
            } else {
#pragma unroll
                for (int j = 0; j < 8; j++)
                    if (n + j < P.N) yp[j] = f2bf(v[j] + (P.bias ? bf2f(P.bias[n + j]) : 0.f));
            }
        }
    }

    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

}  // namespace gm
