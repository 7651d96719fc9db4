// Attention inside many short independent sequences (seq <= 16) on the 5th-generation tensor cores, fed by TMA: the
// DiT passes (11 tokens, all takes x both CFG branches in one launch) and the local encoder (5 tokens) of a decoding
// step (src/model.rs:541-567, kernels/voxcpm.cu:262-297), and any other short-sequence call of attn_full.
//
// Work unit: one sequence and a block of HS q heads with the kv heads they read.
//   grouped heads (G = nq / nk >= 2): HS q heads of one kv head (HS = G when G * seq <= 128), KS = 1 kv head;
//   one q head per kv head (G = 1): HS stacked q heads and their own HS kv heads (KS = HS), the scores of a query
//   against the other heads' keys masked out (so S is block-diagonal in the stacked layout).
// Each unit is three 3-D TMA boxes per 64-column half of hd, over qkv viewed as [rows][heads][hd]:
//   Q {64, HS, seq} -> shared rows m = r * HS + g (query r of q head g), 128-byte swizzled
//   K {64, KS, seq}, V {64, KS, seq} -> shared rows c = r' * KS + h' (key r' of kv head h')
// so a whole unit lands with one barrier, and no byte of qkv is read twice.
//
// Persistent CTAs (one per SM, units strided over the grid), warp roles:
//   warp 0       TMEM allocator and TMA producer: the units' boxes into a ring of NSLOT shared-memory slots
//   warps 4..    NWG warpgroups (3 for grouped heads, 2 for stacked ones), unit k of the CTA to warpgroup k % NWG,
//                each independent of the others: (rope: q and k rotated in shared memory, the arithmetic of k_rope,
//                so the result is bit-identical to rope then attention), then its elected thread issues
//                  S = Q . K^T   (M = 128 rows, N = 16 .. 128 keys, K = hd; both operands K-major, 128-B swizzle)
//                into its TMEM columns; thread m = row m loads its S row, runs the masked softmax in fp32 (exp2
//                with the scale folded in) and writes P back into the S columns as bf16 hi + lo (the weights keep
//                ~16 mantissa bits); the elected thread issues
//                  O = P_hi . V + P_lo . V   (M = 128, N = hd, K = keys; A = P from tensor memory, B = V MN-major)
//                and thread m scales its O row by 1 / sum into bf16 (the reference's normalisation point,
//                kernels/voxcpm.cu:291-295), staged into the unit's slot, from where the elected thread stores the
//                box to the output with TMA.
// TMEM per warpgroup: grouped heads S/P in columns [32w, 32w + 16), O in [128(w + 1), 128(w + 1) + hd); stacked
// heads S/P in [256w, 256w + 128), O in [256w + 128, 256w + 128 + hd).
// All waits are bounded (mbar_wait); on a timeout the kernel records the error and winds down.
#pragma once
#include "common.cuh"

namespace sq {

// warps 0..3 (producer, then idle) and NWG compute warpgroups
__host__ __device__ constexpr int nthreads(int nwg) { return (4 + 4 * nwg) * 32; }
constexpr int NSLOT_MAX = 8;
constexpr int SLACK = 16384;       // the S MMA reads 128 rows from the start of the last Q box of a slot
constexpr int BAR_BYTES = 512;

struct Params {
    const float *cos_t, *sin_t;  // rope tables (ROPE builds)
    int seq, causal, nq, nk, G;
    int HS, KS;                  // q heads and kv heads per unit
    int qrows, krows, ns;        // HS * seq, KS * seq, the S width (krows rounded up to 16)
    int ups, units;              // units per sequence, units in all
    int qbox, kbox, slot, nslot; // bytes: one Q box region, one K (or V) box region, one slot; slots
    float sl2;                   // scale * log2(e)
};

// Shared-memory layout from the 1024-aligned base: NSLOT slots, the slack, the barriers.
enum { B_FULL = 0, B_EMPTY = B_FULL + NSLOT_MAX, B_S = B_EMPTY + NSLOT_MAX, B_O = B_S + 3, B_TMEM = B_O + 3,
       B_ABORT = B_TMEM + 1, B_COUNT = B_ABORT + 1 };
static_assert(B_COUNT * 8 <= BAR_BYTES, "barrier area");

constexpr int TAB_BYTES = 16 * 64 * 4 * 2;  // rope: cos and sin rows of the (at most 16) positions, fp32
__host__ __device__ inline int smem_bytes(int slot, int nslot) {
    return 1024 + nslot * slot + SLACK + BAR_BYTES + TAB_BYTES;
}

// Rotate 8 rope pairs in place: elements [8p, 8p + 8) of the first half of a row (u1) with the same elements of
// the second half (u2), with the table values c, sn of their position: x1' = bf16(x1*c - x2*s), x2' = bf16(x2*c +
// x1*s) in fp32, the expression of k_rope (kernels/voxcpm.cu:109-114).
__device__ __forceinline__ void rope8(uint4 &u1, uint4 &u2, const float (&c)[8], const float (&sn)[8]) {
    // two elements per conversion (cvt.rn.bf16x2.f32): the same round-to-nearest-even, half the conversions
    const uint32_t a[4] = {u1.x, u1.y, u1.z, u1.w}, b[4] = {u2.x, u2.y, u2.z, u2.w};
    uint32_t oa[4], ob[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float2 x1 = unpack_bf16x2(a[j]), x2 = unpack_bf16x2(b[j]);
        const float c0 = c[2 * j], c1 = c[2 * j + 1], s0 = sn[2 * j], s1 = sn[2 * j + 1];
        oa[j] = pack_bf16x2(x1.x * c0 - x2.x * s0, x1.y * c1 - x2.y * s1);
        ob[j] = pack_bf16x2(x2.x * c0 + x1.x * s0, x2.y * c1 + x1.y * s1);
    }
    u1 = make_uint4(oa[0], oa[1], oa[2], oa[3]);
    u2 = make_uint4(ob[0], ob[1], ob[2], ob[3]);
}

// Byte offset of 16-byte chunk `ch` (0 .. hd/8 - 1) of swizzled row `row` in a matrix of boxes `box` bytes apart.
__device__ __forceinline__ uint32_t chunk_off(int row, int ch, int box) {
    return static_cast<uint32_t>((ch >> 3) * box) + sw128(row, ch & 7);
}

__device__ __forceinline__ void ld_shared_v4(uint32_t addr, uint4 &v) {
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
}

// Unit u: sequence n, first q head qh0, first kv head kh0.
__device__ __forceinline__ void unit_heads(const Params &P, int u, int &n, int &qh0, int &kh0) {
    n = u / P.ups;
    const int rem = u - n * P.ups;
    if (P.G > 1) {
        const int sub = P.G / P.HS;
        kh0 = rem / sub;
        qh0 = kh0 * P.G + (rem - kh0 * sub) * P.HS;
    } else {
        qh0 = rem * P.HS;
        kh0 = qh0;
    }
}

// Named barrier of warpgroup w (IDs 1..3) that also ANDs `pred` over its 128 threads.
__device__ __forceinline__ bool wg_and(int w, bool pred) {
    return w == 0 ? bar_and<1, 128>(pred) : (w == 1 ? bar_and<2, 128>(pred) : bar_and<3, 128>(pred));
}

// NMAX: S columns loaded per row (16 for grouped heads, 128 for stacked heads). NWG: compute warpgroups. ROPE: q and
// k rotated in shared memory at position r of the sequence before S.
template <int HD, int NMAX, int NWG, bool ROPE>
__global__ void __launch_bounds__(nthreads(NWG), 1)
    k_attn_small_tc(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tkv,
                    const __grid_constant__ CUtensorMap tout, const Params P) {
    constexpr int NBOX = HD / 64;
    static_assert(NWG * (NMAX == 16 ? 128 : 256) <= 512, "TMEM columns");
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_s = smem_u32(smem_raw);
    uint8_t *sm = smem_raw + ((1024u - (raw_s & 1023u)) & 1023u);
    const uint32_t sm_s = smem_u32(sm);
    const int bar_off = P.nslot * P.slot + SLACK;
    const uint32_t bars = sm_s + bar_off;
    auto bar = [&](int i) { return bars + 8u * i; };
    volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(sm + bar_off + 8 * B_TMEM);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(sm + bar_off + 8 * B_ABORT);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grid = gridDim.x, c = blockIdx.x;
    const int nunits = c < P.units ? (P.units - c + grid - 1) / grid : 0;  // this CTA's units: c, c + grid, ...
    auto slot_s = [&](int k) { return sm_s + static_cast<uint32_t>((k % P.nslot) * P.slot); };
    const int koff = NBOX * P.qbox, voff = koff + NBOX * P.kbox;  // K and V boxes within a slot

    if (threadIdx.x == 0) {
        for (int i = 0; i < NSLOT_MAX; i++) {
            mbar_init(bar(B_FULL + i), 1);
            mbar_init(bar(B_EMPTY + i), 1);
        }
        for (int w = 0; w < 3; w++) {
            mbar_init(bar(B_S + w), 1);
            mbar_init(bar(B_O + w), 1);
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    // Programmatic dependent launch: the set-up above and the padding below overlap the preceding kernel; TMEM is
    // allocated only after it has completed (a kernel that takes all 512 columns before its predecessor ends could
    // hold columns that predecessor has yet to allocate), and the next kernel is let in only once the columns are
    // held (so none of its CTAs can take them first).
    // The producer's first unit goes out as soon as the preceding kernel has completed, ahead of the TMEM allocation
    // and the block-wide set-up (the padding below writes other rows of the slots); the rest once the warpgroups run.
    // (All the slots' units issued that early held the set-up back: 15.2 against 12.1 us at the DiT shape.)
    const uint32_t tx = static_cast<uint32_t>(NBOX * (P.qrows + 2 * P.krows) * 128);
    auto issue = [&](int k) {
        int n, qh0, kh0;
        unit_heads(P, c + k * grid, n, qh0, kh0);
        const uint32_t dst = slot_s(k), fb = bar(B_FULL + k % P.nslot);
        mbar_expect_tx(fb, tx);
#pragma unroll
        for (int b = 0; b < NBOX; b++) {
            tma_load_3d(dst + b * P.qbox, &tq, fb, b * 64, qh0, n * P.seq);
            tma_load_3d(dst + koff + b * P.kbox, &tkv, fb, b * 64, P.nq + kh0, n * P.seq);
            tma_load_3d(dst + voff + b * P.kbox, &tkv, fb, b * 64, P.nq + P.nk + kh0, n * P.seq);
        }
    };
    const int first = nunits < 1 ? nunits : 1;
    int last_k[NSLOT_MAX];  // producer: the last unit loaded into each slot (-1: none)
    if (warp == 0) {
        pdl_wait();
        if (lane == 0) {
            tma_prefetch_desc(&tq);
            tma_prefetch_desc(&tkv);
            tma_prefetch_desc(&tout);
#pragma unroll
            for (int i = 0; i < NSLOT_MAX; i++) last_k[i] = i < first ? i : -1;
            for (int k = 0; k < first; k++) issue(k);
        }
        __syncwarp();
        tmem_alloc(bar(B_TMEM), 512);
        tmem_relinquish();
    }
    // The K and V boxes hold krows rows but the MMAs read ns (a multiple of 16): the rows in between are never
    // loaded, and P = 0 there does not cancel stale shared memory (0 * NaN is NaN), so they are zeroed once.
    {
        const int pad = (P.ns - P.krows) * 8;  // 16-byte chunks per box
        const int items = P.nslot * 2 * NBOX * pad;
        for (int i = threadIdx.x; i < items; i += nthreads(NWG)) {
            const int box = i / pad, ch = i - box * pad;
            const int sl = box / (2 * NBOX), kv = box - sl * 2 * NBOX;
            const uint32_t a = sm_s + static_cast<uint32_t>(sl * P.slot + koff + kv * P.kbox + P.krows * 128 + ch * 16);
            st_shared_v4(a, make_uint4(0u, 0u, 0u, 0u));
        }
        fence_proxy_async_smem();  // read by the tensor cores through the async proxy
    }
    // rope: the cos and sin rows of positions [0, seq) in shared memory, [seq][hd/2] each
    float *tab_c = reinterpret_cast<float *>(sm + bar_off + BAR_BYTES);
    float *tab_s = tab_c + TAB_BYTES / 8;
    if (ROPE) {
        pdl_wait();  // the tables are read after the preceding kernel like every other input
        for (int i = threadIdx.x; i < P.seq * (HD / 2); i += nthreads(NWG)) {
            tab_c[i] = P.cos_t[i];
            tab_s[i] = P.sin_t[i];
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (threadIdx.x == 0) pdl_trigger();

    if (warp == 0) {
        // ------------------------------ TMA producer: the units after the first ------------------------------
        if (lane == 0) {
            for (int k = first; k < nunits; k++) {
                const int s = k % P.nslot;
                if (!mbar_wait(bar(B_EMPTY + s), ((k / P.nslot) - 1) & 1)) {
                    *abort_flag = 1;
                    break;
                }
                if (*abort_flag) break;
                issue(k);
                last_k[s] = k;
            }
        }
        __syncwarp();
    }
    else if (warp >= 4) {
        // ------------------------------ compute warpgroups ------------------------------
        const int w = (warp - 4) >> 2;                     // units k = w, w + NWG, ...
        const int wtid = threadIdx.x - 128 * (1 + w);      // 0 .. 127 within the warpgroup; 0 issues MMAs and stores
        const int m = (warp & 3) * 32 + lane;              // the row of S and O this thread owns (its TMEM lane)
        const uint32_t colSP = NMAX == 16 ? 32u * w : 256u * w;
        const uint32_t colO = NMAX == 16 ? 128u * (w + 1) : 256u * w + 128u;
        const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
        const uint32_t tSP = tmem + lane_off + colSP, tO = tmem + lane_off + colO;
        const int r = m / P.HS, g = m - r * P.HS;          // query position, q head within the unit
        constexpr int GS = NMAX < 32 ? NMAX : 32;          // columns per softmax group
        uint32_t vm[NMAX / GS];                             // visible keys of row m, one bit per column
#pragma unroll
        for (int q = 0; q < NMAX / GS; q++) {
            uint32_t bits = 0;
            for (int i = 0; i < GS; i++) {
                const int col = q * GS + i, kp = col / P.KS, kh = col - kp * P.KS;
                const bool v = m < P.qrows && col < P.krows && (P.KS == 1 || kh == g) && (!P.causal || kp <= r);
                bits |= (v ? 1u : 0u) << i;
            }
            vm[q] = bits;
        }
        const uint32_t idS = idesc_bf16_f32(128, P.ns, 0, 0), idO = idesc_bf16_f32(128, HD, 0, 1);
        int s_issued = -1, o_issued = -1;  // (thread wtid 0) the last unit whose S / P.V it issued
        bool ok = true;
        for (int k = w; k < nunits; k += NWG) {
            const int j = k / NWG;
            const uint32_t base = slot_s(k);
            ok = ok && __all_sync(0xffffffffu, mbar_wait(bar(B_FULL + k % P.nslot), (k / P.nslot) & 1));
            if (ROPE && ok) {
                // q and k rotated in place at their positions in the sequence (v is not), before S reads them;
                // two items (16-byte chunk pairs) per thread at a time: every load is issued before any store
                constexpr int HP = HD / 16;  // chunk p of a row pairs with chunk p + HP (element d with d + hd/2)
                constexpr int NB = 2;
                const int items = (P.qrows + P.krows) * HP;
                for (int it0 = wtid; it0 < items; it0 += NB * 128) {
                    uint4 u1[NB], u2[NB];
                    uint32_t a1[NB], a2[NB];
                    float cv[NB][8], sv[NB][8];
#pragma unroll
                    for (int b = 0; b < NB; b++) {
                        const int it = it0 + b * 128;
                        if (it >= items) continue;
                        const int ri = it / HP, p = it - ri * HP;
                        const bool isq = ri < P.qrows;
                        const int row = isq ? ri : ri - P.qrows;
                        const int pos = isq ? row / P.HS : row / P.KS;
                        const uint32_t mb = isq ? base : base + koff;
                        const int bx = isq ? P.qbox : P.kbox;
                        a1[b] = mb + chunk_off(row, p, bx);
                        a2[b] = mb + chunk_off(row, p + HP, bx);
                        ld_shared_v4(a1[b], u1[b]);
                        ld_shared_v4(a2[b], u2[b]);
                        const float4 *ct = reinterpret_cast<const float4 *>(tab_c + pos * (HD / 2) + p * 8);
                        const float4 *st = reinterpret_cast<const float4 *>(tab_s + pos * (HD / 2) + p * 8);
                        const float4 c0 = ct[0], c1 = ct[1], s0 = st[0], s1 = st[1];
                        cv[b][0] = c0.x; cv[b][1] = c0.y; cv[b][2] = c0.z; cv[b][3] = c0.w;
                        cv[b][4] = c1.x; cv[b][5] = c1.y; cv[b][6] = c1.z; cv[b][7] = c1.w;
                        sv[b][0] = s0.x; sv[b][1] = s0.y; sv[b][2] = s0.z; sv[b][3] = s0.w;
                        sv[b][4] = s1.x; sv[b][5] = s1.y; sv[b][6] = s1.z; sv[b][7] = s1.w;
                    }
#pragma unroll
                    for (int b = 0; b < NB; b++) {
                        if (it0 + b * 128 >= items) continue;
                        rope8(u1[b], u2[b], cv[b], sv[b]);
                        st_shared_v4(a1[b], u1[b]);
                        st_shared_v4(a2[b], u2[b]);
                    }
                }
                fence_proxy_async_smem();  // the tensor cores read these rows through the async proxy
            }
            ok = wg_and(w, ok);
            if (!ok) break;
            if (wtid == 0) {  // S = Q . K^T
                tc_fence_after();
#pragma unroll
                for (int ks = 0; ks < HD / 16; ks++) {
                    const uint64_t a = smem_desc_sw128(base + (ks >> 2) * P.qbox + (ks & 3) * 32, 16, 1024);
                    const uint64_t b = smem_desc_sw128(base + koff + (ks >> 2) * P.kbox + (ks & 3) * 32, 16, 1024);
                    tc_mma_ss(tmem + colSP, a, b, idS, ks > 0 ? 1u : 0u);
                }
                tc_commit(bar(B_S + w));
                s_issued = j;
                // while S runs: the previous unit's output stores have read their slot, which goes back to the
                // producer (nothing waits for it on the unit's own chain)
                if (k >= w + NWG) {
                    bulk_wait_read();
                    mbar_arrive(bar(B_EMPTY + (k - NWG) % P.nslot));
                }
            }
            __syncwarp();
            // ---- softmax of row m: S from TMEM, P (bf16 hi + lo) back into the same columns ----
            ok = __all_sync(0xffffffffu, mbar_wait(bar(B_S + w), j & 1));
            float inv = 0.f;
            if (ok) {
                tc_fence_after();
                uint32_t sr[NMAX];
                if constexpr (NMAX == 16) {
                    tmem_ld16(tSP, sr);
                } else {
#pragma unroll
                    for (int q = 0; q < NMAX / 32; q++) tmem_ld32(tSP + 32 * q, sr + 32 * q);
                }
                tc_wait_ld();
                float mx = -INFINITY;
#pragma unroll
                for (int col = 0; col < NMAX; col++) {
                    const float sv = (vm[col / GS] >> (col % GS)) & 1u ? __uint_as_float(sr[col]) * P.sl2 : -INFINITY;
                    sr[col] = __float_as_uint(sv);
                    mx = fmaxf(mx, sv);
                }
                if (mx == -INFINITY) mx = 0.f;  // rows past the unit (or a row with no visible key)
                float sum = 0.f;
#pragma unroll
                for (int q = 0; q < NMAX / GS; q++) {
                    uint32_t hw[GS / 2], lw[GS / 2];
#pragma unroll
                    for (int i = 0; i < GS / 2; i++) {
                        const float p0 = fast_exp2(__uint_as_float(sr[q * GS + 2 * i]) - mx);
                        const float p1 = fast_exp2(__uint_as_float(sr[q * GS + 2 * i + 1]) - mx);
                        sum += p0 + p1;
                        hw[i] = pack_bf16x2(p0, p1);
                        const float2 hv = unpack_bf16x2(hw[i]);
                        lw[i] = pack_bf16x2(p0 - hv.x, p1 - hv.y);
                    }
                    if constexpr (GS == 16) {
                        tmem_st8(tSP + q * 8, hw);
                        tmem_st8(tSP + NMAX / 2 + q * 8, lw);
                    } else {
                        tmem_st16(tSP + q * 16, hw);
                        tmem_st16(tSP + NMAX / 2 + q * 16, lw);
                    }
                }
                tc_wait_st();
                inv = 1.f / sum;
            }
            tc_fence_before();
            ok = wg_and(w, ok);
            if (!ok) break;
            if (wtid == 0) {  // O = P_hi . V + P_lo . V
                tc_fence_after();
                const uint32_t vb = base + voff;
                for (int kk = 0; kk < P.ns / 16; kk++) {
                    const uint64_t b = smem_desc_sw128(vb + kk * 2048, P.kbox, 1024);
                    tc_mma_ts(tmem + colO, tmem + colSP + kk * 8, b, idO, kk > 0 ? 1u : 0u);
                    tc_mma_ts(tmem + colO, tmem + colSP + NMAX / 2 + kk * 8, b, idO, 1u);
                }
                tc_commit(bar(B_O + w));
                o_issued = j;
            }
            __syncwarp();
            // ---- epilogue: row m of O, times 1 / sum, as bf16 into the slot's Q boxes (the output box layout) ----
            ok = __all_sync(0xffffffffu, mbar_wait(bar(B_O + w), j & 1));
            if (ok) {
                tc_fence_after();
                // two loads in flight per wait, except in the rope build (which would spill at 128 registers)
                constexpr int OB = ROPE ? 32 : 64;
#pragma unroll
                for (int cb = 0; cb < HD; cb += OB) {
                    uint32_t o[OB];
                    tmem_ld32(tO + cb, o);
                    if (OB == 64 && cb + 32 < HD) tmem_ld32(tO + cb + 32, o + OB - 32);
                    tc_wait_ld();
                    if (m < P.qrows) {
#pragma unroll
                        for (int q = 0; q < OB / 8; q++) {
                            if (cb + q * 8 >= HD) break;
                            uint4 v;
                            v.x = pack_bf16x2(__uint_as_float(o[8 * q]) * inv, __uint_as_float(o[8 * q + 1]) * inv);
                            v.y = pack_bf16x2(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv);
                            v.z = pack_bf16x2(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv);
                            v.w = pack_bf16x2(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv);
                            st_shared_v4(base + chunk_off(m, cb / 8 + q, P.qbox), v);
                        }
                    }
                }
                fence_proxy_async_smem();  // the TMA store reads the staged rows through the async proxy
            }
            tc_fence_before();
            ok = wg_and(w, ok);
            if (!ok) break;
            if (wtid == 0) {
                int n, qh0, kh0;
                unit_heads(P, c + k * grid, n, qh0, kh0);
#pragma unroll
                for (int b = 0; b < NBOX; b++) tma_store_3d(&tout, base + b * P.qbox, b * 64, qh0, n * P.seq);
                bulk_commit();  // the slot goes back to the producer at the next unit, once the stores have read it
            }
            __syncwarp();
        }
        if (wtid == 0) bulk_wait_read();  // every store has read its slot before the CTA may leave
        if (!ok && wtid == 0) {
            *abort_flag = 1;
            // nothing may still write TMEM when it is freed: wait (bounded) for the last MMAs issued
            if (s_issued >= 0) mbar_wait(bar(B_S + w), s_issued & 1);
            if (o_issued >= 0) mbar_wait(bar(B_O + w), o_issued & 1);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
        if (lane == 0 && *abort_flag) {
            // after an abort a load may still be landing: it must not write shared memory of a CTA that has left
            for (int i = 0; i < NSLOT_MAX; i++)
                if (i < P.nslot && last_k[i] >= 0) mbar_wait(bar(B_FULL + i), (last_k[i] / P.nslot) & 1);
        }
    }
}

}  // namespace sq
