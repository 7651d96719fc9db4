// Flash attention for long sequences on the 5th-generation tensor cores (tcgen05 + TMEM), fed by TMA, with two query
// tiles per CTA whose softmax phases alternate (ping-pong): while one warpgroup exponentiates its tile's scores, the
// tensor cores run the other tile's P.V and next S. The same attention as pf::k_attn_prefill (src/model.rs:688,701
// -> full(..., causal); kernels/voxcpm.cu:262-297), for prompts long enough that every SM holds such a pair.
//
// One CTA per (q head, pair of consecutive 128-query tiles A = 2p and B = 2p + 1, sequence), heaviest pairs first.
// Warp roles:
//   warp 0      TMA producer: Q_A and Q_B once, then K and V tiles of 128 positions into two 2-stage rings (the V
//               loads trailing the K loads by one tile); a stage is reused once both tiles' MMAs have read it
//   warp 1      TMEM allocator and the single MMA-issuing thread, in the order
//                 S_A(0) S_B(0) | PV_A(0) S_A(1) PV_B(0) S_B(1) | PV_A(1) S_A(2) PV_B(1) S_B(2) | ...
//               so S_A(j+1) and PV_B(j) run under warpgroup A's softmax of tile j+1, and the other way round
//   warps 2..5  softmax of tile A, warps 6..9 of tile B: thread = one query row, all 128 key columns of it. Pass 1
//               takes the row max over S (lazy rescaling as in pf::k_attn_prefill: the stale max stays unless the
//               new one exceeds it by more than 2^8); pass 2 exponentiates each 32-column quarter and writes it back
//               into the same TMEM columns as P (hi: p truncated to bf16; lo: the rest rounded,
//               ~16 bits of p in all), so P aliases S. The row sum stays in the thread; at the end O / sum -> bf16.
// TMEM (512 columns): S/P of A [0, 128), S/P of B [128, 256), O of A [256, 256 + hd), O of B [384, 384 + hd).
// Keys 32q .. 32q + 31 of P sit in columns 32q + [0, 16) (hi pairs) and 32q + [16, 32) (lo pairs): quarter q of the
// row is written only where quarter q of S was, after it has been read. The next S of a tile overwrites its P, so it is
// issued once that tile's P.V has completed.
// All waits are bounded (mbar_wait); on a timeout the kernel records the error and winds down.
#pragma once
#include "common.cuh"
#include "prefill_tc.cuh"  // pf::exp2_poly2

namespace pp {

constexpr int BM = 128, BN = 128;
constexpr int NTHREADS = 10 * 32;   // TMA, MMA, two softmax warpgroups
constexpr float RESCALE_LOG2 = 8.f;
constexpr int BOX = 128 * 128;      // one 128-row x 128-byte swizzled box

template <int HD>
struct Cfg {
    static constexpr int NBOX = HD / 64;
    static constexpr int QA_OFF = 0;
    static constexpr int QB_OFF = QA_OFF + NBOX * BOX;
    static constexpr int K_OFF = QB_OFF + NBOX * BOX;      // 2 stages
    static constexpr int V_OFF = K_OFF + 2 * NBOX * BOX;   // 2 stages
    static constexpr int BAR_OFF = V_OFF + 2 * NBOX * BOX;
    static constexpr int SMEM = BAR_OFF + 256 + 1024;      // + alignment slack
    static constexpr uint32_t TMEM_COLS = 512;
    // tile x: S/P in columns [128x, 128x + 128), O in [256 + 128x, 256 + 128x + hd)
    __host__ __device__ static constexpr uint32_t s_col(int x) { return 128u * x; }
    __host__ __device__ static constexpr uint32_t o_col(int x) { return 256u + 128u * x; }
};

enum { B_Q = 0, B_KF0 = 1, B_KF1 = 2, B_KE0 = 3, B_KE1 = 4, B_VF0 = 5, B_VF1 = 6, B_VE0 = 7, B_VE1 = 8,
       B_SFULL0 = 9, B_SFULL1 = 10, B_PFULL0 = 11, B_PFULL1 = 12, B_PVD0 = 13, B_PVD1 = 14, B_TMEM = 15,
       B_ABORT = 16, B_COUNT = 17 };
static_assert(B_COUNT * 8 <= 256, "barrier area");

template <int HD>
__global__ void __launch_bounds__(NTHREADS, 1)
    k_attn_prefill_pp(const __grid_constant__ CUtensorMap tqkv, bf16 *__restrict__ out, int seq, int causal, int nq,
                      int nk, float sl2) {
    using C = Cfg<HD>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_s = smem_u32(smem_raw);
    uint8_t *sm = smem_raw + ((1024u - (raw_s & 1023u)) & 1023u);
    const uint32_t sm_s = smem_u32(sm);
    const uint32_t bars = sm_s + C::BAR_OFF;
    auto bar = [&](int i) { return bars + 8u * i; };
    volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(sm + C::BAR_OFF + 8 * B_TMEM);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(sm + C::BAR_OFF + 8 * B_ABORT);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qtiles = (seq + BM - 1) / BM;
    const int pr = gridDim.y - 1 - blockIdx.y;  // heaviest pairs first
    const int h = blockIdx.x, n = blockIdx.z, kh = h / (nq / nk);
    const int row0 = n * seq;
    const int ntiles_all = (seq + BN - 1) / BN;
    // query tile x = 2 pr + x and the key tiles it attends over (0: no such tile)
    auto ntiles_of = [&](int x) {
        const int q = 2 * pr + x;
        return q >= qtiles ? 0 : (causal ? min(ntiles_all, (q * BM + BM - 1) / BN + 1) : ntiles_all);
    };
    const int nt0 = ntiles_of(0), nt1 = ntiles_of(1);
    const int nmax = nt0 > nt1 ? nt0 : nt1;

    if (threadIdx.x == 0) {
        for (int i = 0; i < B_TMEM; i++) mbar_init(bar(i), (i == B_PFULL0 || i == B_PFULL1) ? 4 : 1);
        *abort_flag = 0;
        mbar_fence_init();
    }
    // Programmatic dependent launch: set-up overlaps the preceding kernel; TMEM is allocated only once it has
    // completed, and the next kernel is let in only once the columns are held (as in pf::k_attn_prefill).
    if (warp == 1) {
        pdl_wait();
        tmem_alloc(bar(B_TMEM), C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (threadIdx.x == 0) pdl_trigger();

    if (warp == 0) {
        // ------------------------------ TMA producer ------------------------------
        if (lane == 0) {
            tma_prefetch_desc(&tqkv);
            mbar_expect_tx(bar(B_Q), (nt1 > 0 ? 2 : 1) * C::NBOX * BOX);
#pragma unroll
            for (int x = 0; x < 2; x++) {
                if ((x ? nt1 : nt0) == 0) continue;
#pragma unroll
                for (int bx = 0; bx < C::NBOX; bx++)
                    tma_load_2d(sm_s + (x ? C::QB_OFF : C::QA_OFF) + bx * BOX, &tqkv, bar(B_Q), h * HD + bx * 64,
                                row0 + (2 * pr + x) * BM);
            }
            auto load_half = [&](int v, int stg, int tj) {
                const uint32_t fb = bar((v ? B_VF0 : B_KF0) + stg);
                mbar_expect_tx(fb, C::NBOX * BOX);
#pragma unroll
                for (int bx = 0; bx < C::NBOX; bx++)
                    tma_load_2d(sm_s + (v ? C::V_OFF : C::K_OFF) + (stg * C::NBOX + bx) * BOX, &tqkv, fb,
                                (nq + (v ? nk : 0) + kh) * HD + bx * 64, row0 + tj * BN);
            };
            bool ok = true;
            int lastk0 = -1, lastk1 = -1, lastv0 = -1, lastv1 = -1;  // the last tile loaded into each stage
            // K0, K1, V0, K2, V1, ...: a K stage waits only for the S MMAs of the tile two back
            for (int j = 0; ok && j <= nmax; j++) {
                if (j < nmax) {
                    if (j >= 2) ok = mbar_wait(bar(B_KE0 + (j & 1)), ((j >> 1) - 1) & 1);
                    if (!ok || *abort_flag) break;
                    load_half(0, j & 1, j);
                    if (j & 1) lastk1 = j; else lastk0 = j;
                }
                if (j >= 1) {
                    const int v = j - 1;
                    if (v >= 2) ok = mbar_wait(bar(B_VE0 + (v & 1)), ((v >> 1) - 1) & 1);
                    if (!ok || *abort_flag) break;
                    load_half(1, v & 1, v);
                    if (v & 1) lastv1 = v; else lastv0 = v;
                }
            }
            if (!ok) *abort_flag = 1;
            if (*abort_flag) {
                // the consumers no longer wait for every load: wait (bounded) until each one issued has landed, since
                // a copy must not write the shared memory of a CTA that has left
                mbar_wait(bar(B_Q), 0);
                if (lastk0 >= 0) mbar_wait(bar(B_KF0), (lastk0 >> 1) & 1);
                if (lastk1 >= 0) mbar_wait(bar(B_KF1), (lastk1 >> 1) & 1);
                if (lastv0 >= 0) mbar_wait(bar(B_VF0), (lastv0 >> 1) & 1);
                if (lastv1 >= 0) mbar_wait(bar(B_VF1), (lastv1 >> 1) & 1);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------ MMA issuer ------------------------------
        if (lane == 0) {
            const uint32_t idS = idesc_bf16_f32(BM, BN, 0, 0);
            const uint32_t idO = idesc_bf16_f32(BM, HD, 0, 1);
            bool ok = mbar_wait(bar(B_Q), 0);
            // the shared-memory base read afresh per call, so that the descriptors of every stage and tile are not
            // all kept live across the loop (registers are shared with the softmax warps' far larger needs)
            auto fresh = [&]() {
                uint32_t b;
                asm volatile("mov.u32 %0, %1;" : "=r"(b) : "r"(sm_s));
                return b;
            };
            auto issue_S = [&](int x, int j) {  // S_x(j) = Q_x . K_j^T into S_x's columns
                const uint32_t base = fresh();
                const uint32_t kbase = base + C::K_OFF + (j & 1) * C::NBOX * BOX;
                const uint32_t qbase = base + (x ? C::QB_OFF : C::QA_OFF);
#pragma unroll
                for (int ks = 0; ks < HD / 16; ks++) {
                    const uint64_t a = smem_desc_sw128(qbase + (ks >> 2) * BOX + (ks & 3) * 32, 16, 1024);
                    const uint64_t b = smem_desc_sw128(kbase + (ks >> 2) * BOX + (ks & 3) * 32, 16, 1024);
                    tc_mma_ss(tmem + C::s_col(x), a, b, idS, ks > 0 ? 1u : 0u);
                }
                tc_commit(bar(B_SFULL0 + x));
            };
            auto issue_PV = [&](int x, int j) {  // O_x += P_x(j) . V_j, hi and lo halves of P from S_x's columns
                const uint32_t vbase = fresh() + C::V_OFF + (j & 1) * C::NBOX * BOX;
#pragma unroll
                for (int kk = 0; kk < BN / 16; kk++) {
                    const uint64_t b = smem_desc_sw128(vbase + kk * 2048, BOX, 1024);
                    const uint32_t tp = tmem + C::s_col(x) + (kk >> 1) * 32 + (kk & 1) * 8;
                    tc_mma_ts(tmem + C::o_col(x), tp, b, idO, (j > 0 || kk > 0) ? 1u : 0u);
                    tc_mma_ts(tmem + C::o_col(x), tp + 16, b, idO, 1u);
                }
                tc_commit(bar(B_PVD0 + x));
            };
            // prologue: both tiles' first S
            if (ok && nmax > 0) {
                ok = mbar_wait(bar(B_KF0), 0);
                if (ok) {
                    tc_fence_after();
                    issue_S(0, 0);
                    if (nt1 > 0) issue_S(1, 0);
                    tc_commit(bar(B_KE0));
                }
            }
            for (int j = 0; ok && j < nmax; j++) {
                bool kwaited = false;  // K_{j+1} has landed (waited once)
#pragma unroll
                for (int x = 0; x < 2; x++) {
                    const int ntx = x ? nt1 : nt0;
                    if (!ok || j >= ntx) continue;
                    // P_x(j) written and V_j landed
                    ok = mbar_wait(bar(B_PFULL0 + x), j & 1) && mbar_wait(bar(B_VF0 + (j & 1)), (j >> 1) & 1);
                    if (!ok) continue;
                    tc_fence_after();
                    issue_PV(x, j);
                    if (j + 1 < ntx) {
                        // S_x(j+1) overwrites P_x(j): only once P_x(j).V has completed
                        ok = mbar_wait(bar(B_PVD0 + x), j & 1) &&
                             (kwaited || mbar_wait(bar(B_KF0 + ((j + 1) & 1)), ((j + 1) >> 1) & 1));
                        if (!ok) continue;
                        kwaited = true;
                        tc_fence_after();
                        issue_S(x, j + 1);
                    }
                }
                if (!ok) break;
                tc_commit(bar(B_VE0 + (j & 1)));                 // V_j: both P.V issued before this commit
                if (j + 1 < nmax) tc_commit(bar(B_KE0 + ((j + 1) & 1)));  // K_{j+1}: both S issued
            }
            if (!ok) *abort_flag = 1;
        }
        __syncwarp();
    } else {
        // ------------------------------ softmax / correction / epilogue ------------------------------
        const int x = (warp - 2) >> 2;      // the tile of this warpgroup
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;  // query row within the tile
        const int q0 = (2 * pr + x) * BM, qrow = q0 + r;
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        const uint32_t tS = tmem + lane_off + C::s_col(x), tO = tmem + lane_off + C::o_col(x);
        const int ntx = x ? nt1 : nt0;
        // the row sum in two halves (keys 0..63 and 64..127 of every tile), each summed as pf::k_attn_prefill's
        // warpgroup for those columns sums it, so that the output is bit-identical to that kernel's
        float m = -INFINITY, l0 = 0.f, l1 = 0.f;
        bool ok = true;
        for (int j = 0; j < ntx; j++) {
            ok = ok && __all_sync(0xffffffffu, mbar_wait(bar(B_SFULL0 + x), j & 1));
            if (!ok) break;
            tc_fence_after();
            const int kbase = j * BN;
            const bool masked = (causal && kbase + BN - 1 > q0) || kbase + BN > seq;
            const int kmax = (causal ? min(seq, qrow + 1) : seq) - kbase;
            // pass 1: the row max, 64 columns (two loads in flight) at a time
            float mh = -INFINITY;
#pragma unroll
            for (int c = 0; c < 2; c++) {
                uint32_t sr[64];
                tmem_ld32(tS + 64 * c, sr);
                tmem_ld32(tS + 64 * c + 32, sr + 32);
                tc_wait_ld();
                if (masked) {
#pragma unroll
                    for (int k = 0; k < 64; k++)
                        if (64 * c + k >= kmax) sr[k] = __float_as_uint(-INFINITY);
                }
                float mt4[4];
#pragma unroll
                for (int k = 0; k < 4; k++) mt4[k] = -INFINITY;
#pragma unroll
                for (int k = 0; k < 64; k += 2)
                    mt4[(k >> 1) & 3] = fmax3(mt4[(k >> 1) & 3], __uint_as_float(sr[k]), __uint_as_float(sr[k + 1]));
                mh = fmax3(mh, fmax3(mt4[0], mt4[1], mt4[2]), mt4[3]);
            }
            const float mt = mh * sl2;
            float alpha = 1.f;
            if (mt > m + RESCALE_LOG2) {
                alpha = fast_exp2(m - mt);  // 0 on the first tile (m = -inf)
                m = mt;
            }
            const float mref = m == -INFINITY ? 0.f : m;
            const float2 sl2v = make_float2(sl2, sl2), nmref = make_float2(-mref, -mref);
            float2 rsa[4], rsb[4];  // the sum chains of keys 0..63 and of keys 64..127
#pragma unroll
            for (int k = 0; k < 4; k++) rsa[k] = rsb[k] = make_float2(0.f, 0.f);
            // pass 2: each quarter exponentiated and written back as P into its own 32 columns (hi pairs, then lo);
            // one pair in eight on the FMA pipe (pf::exp2_poly2), the same pairs as pf::k_attn_prefill
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
            float2 (&rs)[4] = hh ? rsb : rsa;
#pragma unroll 1
            for (int q = 2 * hh; q < 2 * hh + 2; q++) {
                uint32_t sr[32], hw[16], lw[16];
                tmem_ld32(tS + 32 * q, sr);
                tc_wait_ld();
                if (masked) {
#pragma unroll
                    for (int k = 0; k < 32; k++)
                        if (32 * q + k >= kmax) sr[k] = __float_as_uint(-INFINITY);
                }
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    const float2 xx = fma2(make_float2(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1])),
                                           sl2v, nmref);
                    const float2 p = (i % 8) == 0 ? pf::exp2_poly2(xx) : make_float2(fast_exp2(xx.x), fast_exp2(xx.y));
                    rs[i & 3] = add2(rs[i & 3], p);
                    const uint32_t u0 = __float_as_uint(p.x), u1 = __float_as_uint(p.y);
                    const float2 lo = sub2(p, make_float2(__uint_as_float(u0 & 0xffff0000u),
                                                          __uint_as_float(u1 & 0xffff0000u)));
                    lw[i] = pack_bf16x2(lo.x, lo.y);
                    hw[i] = __byte_perm(u0, u1, 0x7632);
                }
                tmem_st16(tS + 32 * q, hw);
                tmem_st16(tS + 32 * q + 16, lw);
            }
            }
            l0 = l0 * alpha + (((rsa[0].x + rsa[0].y) + (rsa[1].x + rsa[1].y)) +
                               ((rsa[2].x + rsa[2].y) + (rsa[3].x + rsa[3].y)));
            l1 = l1 * alpha + (((rsb[0].x + rsb[0].y) + (rsb[1].x + rsb[1].y)) +
                               ((rsb[2].x + rsb[2].y) + (rsb[3].x + rsb[3].y)));
            // O is rescaled before P_x(j).V adds to it; P_x(j-1).V has completed (S_x(j) was issued after it)
            if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
                for (int c = 0; c < HD; c += 32) {
                    uint32_t orow[32];
                    tmem_ld32(tO + c, orow);
                    tc_wait_ld();
#pragma unroll
                    for (int k = 0; k < 32; k++) orow[k] = __float_as_uint(__uint_as_float(orow[k]) * alpha);
                    tmem_st32(tO + c, orow);
                }
            }
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(B_PFULL0 + x));
        }
        // O is final once the last P.V has completed (the phase before it was waited for through S)
        if (ok && ntx > 0) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_PVD0 + x), (ntx - 1) & 1));
        if (!ok) *abort_flag = 1;
        if (ok && ntx > 0) {
            tc_fence_after();
            const float inv = 1.f / (l0 + l1);
            bf16 *dst = out + static_cast<long>(row0 + qrow) * nq * HD + h * HD;
#pragma unroll 1
            for (int c = 0; c < HD; c += 32) {
                uint32_t orow[32];
                tmem_ld32(tO + c, orow);
                tc_wait_ld();
                if (qrow < seq) {
#pragma unroll
                    for (int k = 0; k < 32; k += 8) {
                        uint4 v;
                        v.x = pack_bf16x2(__uint_as_float(orow[k]) * inv, __uint_as_float(orow[k + 1]) * inv);
                        v.y = pack_bf16x2(__uint_as_float(orow[k + 2]) * inv, __uint_as_float(orow[k + 3]) * inv);
                        v.z = pack_bf16x2(__uint_as_float(orow[k + 4]) * inv, __uint_as_float(orow[k + 5]) * inv);
                        v.w = pack_bf16x2(__uint_as_float(orow[k + 6]) * inv, __uint_as_float(orow[k + 7]) * inv);
                        *reinterpret_cast<uint4 *>(dst + c + k) = v;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

}  // namespace pp
