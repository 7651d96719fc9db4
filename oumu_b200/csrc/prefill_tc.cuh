// Flash attention on the 5th-generation tensor cores (tcgen05 + TMEM), fed by TMA, for long sequences: the causal
// prefill over the prompt (src/model.rs:688,701 -> full(..., causal = true)).
//
// One CTA per (q head, 128-query tile, sequence), heaviest tiles first. Warp roles:
//   warp 0      TMA producer: Q tile once, then K and V tiles of 128 positions into two 2-stage rings: a K stage is
//               free again once its S = Q.K^T has completed, a V stage once its P.V has, so the K of tile j+2
//               loads while P_j.V still runs (the V loads trail the K loads by one tile)
//   warp 1      TMEM allocator and the single MMA-issuing thread:
//                 S  = Q . K_j^T      (M=128 queries, N=128 keys, K=hd; A and B K-major, 128-B swizzle)
//                 O += P_j . V_j      (M=128, N=hd, K=128 keys; A = P from tensor memory, B = V MN-major)
//   warps 2..9  softmax, two warpgroups: warpgroup g owns columns [64g, 64g+64) of every row (thread = row of its
//               TMEM lane quarter). Each thread loads its 64 columns of S from TMEM in one batch and takes their
//               max; the two half-row maxima meet in shared memory at a per-tile barrier of the two warpgroups
//               (which also votes on whether every wait succeeded, so the loop is left uniformly). It then
//               exponentiates its 64 columns, keeps its half of the row sum and writes its half of P_j into TMEM
//               as two bf16 matrices hi + lo (hi truncated, lo the rounded remainder: ~16 mantissa bits;
//               O += P_hi.V + P_lo.V), in one of two P buffers: P_{j+1} is written while P_j.V runs, and a buffer
//               is reused once the P.V two tiles back has read it. It rescales its half of the O row in TMEM when
//               the max has grown by more than 2^8 (lazy rescaling: until then the stale max is kept, which changes
//               no result because O and the sum use the same one). The halves of the sum meet once, at the end,
//               and each warpgroup writes bf16(O * (1 / sum)) for its 64 columns.
// KV epilogue (oumu_attn_prefill_kv, slots > 0): the prompt's k and v also go into every take's cache slot, with TMA
// tensor stores from the 128-byte-swizzled tiles in shared memory through a map whose extent is the prompt length (rows
// past it are never written). The CTA of query tile qt copies key tile ntiles - 1 - qt, the G q heads of a kv head
// splitting the slots: the longest CTAs (late query tiles) copy early key tiles right after loading them, under the
// rest of their math; the shortest ones load and copy the late tiles after their own few tiles.
// All waits are bounded (mbar_wait); on a timeout the kernel records the error and winds down.
#pragma once
#include "common.cuh"

namespace pf {
// 2^x for two lanes on the FMA pipe: x = j + f with j = round(x) (added to and taken from 1.5 * 2^23, whose low
// mantissa bits then hold j) and f in [-1/2, 1/2]; 2^f by a degree-4 polynomial fitted here to 2^f in relative error
// (max 2.6e-6); 2^j added to the exponent bits. x below -126 gives a value below 2^-125 instead of 0.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
    x.x = fmaxf(x.x, -126.f);
    x.y = fmaxf(x.y, -126.f);
    const float2 mg = make_float2(12582912.f, 12582912.f);
    const float2 t = add2(x, mg);
    const float2 f = sub2(x, sub2(t, mg));
    float2 p = fma2(f, make_float2(0.009570096619427204f, 0.009570096619427204f),
                    make_float2(0.05591785907745361f, 0.05591785907745361f));
    p = fma2(p, f, make_float2(0.240247443318367f, 0.240247443318367f));
    p = fma2(p, f, make_float2(0.6931217908859253f, 0.6931217908859253f));
    p = fma2(p, f, make_float2(0.9999992847442627f, 0.9999992847442627f));
    return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                       __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int NTHREADS = 10 * 32;  // TMA, MMA, two softmax warpgroups
constexpr float RESCALE_LOG2 = 8.f;  // O and the sum are rescaled only when the row max grows by more than 2^8
constexpr int BOX = 128 * 128;  // one 128-row x 128-byte swizzled box

template <int HD>
struct Cfg {
    static constexpr int NBOX = HD / 64;
    static constexpr int Q_OFF = 0;
    static constexpr int K_OFF = Q_OFF + NBOX * BOX;         // 2 stages
    static constexpr int V_OFF = K_OFF + 2 * NBOX * BOX;     // 2 stages
    static constexpr int BAR_OFF = V_OFF + 2 * NBOX * BOX;
    static constexpr int LX_OFF = BAR_OFF + 256;             // the two halves of the row sums, 2 x 128 floats
    static constexpr int MX_OFF = LX_OFF + 1024;             // half-row maxima, [tile parity][warpgroup][128]
    static constexpr int SMEM = MX_OFF + 2048 + 1024;        // + alignment slack
    // TMEM: S (128 columns), two P buffers (hi: 64 columns of bf16 pairs, lo: 64), O (hd columns)
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr uint32_t P_COL = 128, O_COL = 384;
};

// barrier slots (8 bytes each) inside the barrier area
enum { B_Q = 0, B_KF0 = 1, B_KF1 = 2, B_KE0 = 3, B_KE1 = 4, B_SFULL = 5, B_SFREE = 6, B_PFULL = 7, B_ODONE = 8,
       B_COPY = 9, B_PDONE0 = 10, B_PDONE1 = 11, B_TMEM = 12, B_ABORT = 13, B_VF0 = 14, B_VF1 = 15, B_VE0 = 16,
       B_VE1 = 17, B_COPY1 = 18 };

// Planned KV epilogue: who copies which part of the prompt's k and v into the slots. Without a plan (planned = 0)
// the CTA of query tile qt copies key tile ntiles - 1 - qt into its q head's share of the slots. With one, the grid
// has one more row (blockIdx.y = 0) of copy CTAs that only copy, a q head's share of the slots is cut into groups of
// gs slots, and group sg of key tile t goes to query tile owner[t][sg] or to the copy CTA (owner = the number of
// query tiles). A CTA copies the groups of the key tiles it loads for its attention as soon as they land (the host
// gives it at most a few per tile, so the wait for those stores to have read the stage before it is reloaded is
// short), and loads the other key tiles it owns groups of after its attention. The host plans so that the longest
// causal query tiles, which bound the kernel, copy nothing while they compute, and no SM stores much more than its
// share: one SM writes only ~85 GB/s with TMA stores.
constexpr int PLAN_MAX = 32, PLAN_GROUPS = 8;
struct CopyPlan {
    int planned, gs;
    signed char owner[PLAN_MAX][PLAN_GROUPS];
};

template <int HD>
__global__ void __launch_bounds__(NTHREADS, 1)
    k_attn_prefill(const __grid_constant__ CUtensorMap tqkv, bf16 *__restrict__ out, int seq, int causal, int nq,
                   int nk, float sl2, const __grid_constant__ CUtensorMap tkc,
                   const __grid_constant__ CUtensorMap tvc, int slots, const __grid_constant__ CopyPlan plan) {
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
    // CTAs start in block order, x fastest: every head's heaviest causal tile first, then the next heaviest, ... so
    // that the tiles left for the last wave are the short ones. A planned KV epilogue puts the copy CTAs first
    // (blockIdx.y = 0, qt = the number of query tiles).
    const bool planned = slots > 0 && plan.planned != 0;
    const bool copier = planned && blockIdx.y == 0;
    const int qt = gridDim.y - 1 - blockIdx.y;
    const int h = blockIdx.x, n = blockIdx.z, G = nq / nk, kh = h / G;
    const int q0 = qt * BM;
    const int row0 = n * seq;  // first row of this sequence in qkv
    const int ntiles_all = (seq + BN - 1) / BN;
    const int ntiles = causal ? min(ntiles_all, (q0 + BM - 1) / BN + 1) : ntiles_all;

    if (threadIdx.x == 0) {
        mbar_init(bar(B_Q), 1);
        mbar_init(bar(B_KF0), 1);
        mbar_init(bar(B_KF1), 1);
        mbar_init(bar(B_KE0), 1);
        mbar_init(bar(B_KE1), 1);
        mbar_init(bar(B_VF0), 1);
        mbar_init(bar(B_VF1), 1);
        mbar_init(bar(B_VE0), 1);
        mbar_init(bar(B_VE1), 1);
        mbar_init(bar(B_SFULL), 1);
        mbar_init(bar(B_SFREE), 8);
        mbar_init(bar(B_PFULL), 8);
        mbar_init(bar(B_ODONE), 1);
        mbar_init(bar(B_COPY), 1);
        mbar_init(bar(B_COPY1), 1);
        mbar_init(bar(B_PDONE0), 1);
        mbar_init(bar(B_PDONE1), 1);
        *abort_flag = 0;
        mbar_fence_init();
    }
    // Programmatic dependent launch: the set-up above overlaps the preceding kernel; TMEM is allocated only after it
    // has completed (a kernel that takes all 512 columns before its predecessor ends could hold columns that
    // predecessor has yet to allocate), and the next kernel is let in only once the columns are held.
    if (warp == 1 && !copier) {
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
        // Lane 0 issues the loads; the KV epilogue's stores are spread over the warp's 32 lanes (one thread keeps
        // only a few bulk copies in flight). Every wait is taken by the whole warp, so control flow stays uniform.
        if (copier) pdl_wait();  // the copy CTAs allocate no TMEM, so no other thread of theirs has waited
        if (lane == 0) {
            tma_prefetch_desc(&tqkv);
            if (!copier) {
                mbar_expect_tx(bar(B_Q), C::NBOX * BOX);
#pragma unroll
                for (int bx = 0; bx < C::NBOX; bx++)
                    tma_load_2d(sm_s + C::Q_OFF + bx * BOX, &tqkv, bar(B_Q), h * HD + bx * 64, row0 + q0);
            }
        }
        // this CTA's share of the KV epilogue: key tile cj (or the plan's tiles) of kv head kh into slots [s0, s1)
        const int cj = ntiles_all - 1 - qt, g = h % G;
        const int per = slots > 0 ? (slots + G - 1) / G : 0, s0 = g * per, s1 = min(slots, s0 + per);
        const bool copy = !planned && slots > 0 && causal && s0 < s1;
        // K (v = 0) or V (v = 1) of key tile tj into stage stg, completing its bytes on barrier fb. tx > 0: this call
        // is the barrier's one arrival, expecting tx bytes; tx == 0: the bytes count against an earlier expectation.
        auto load_half = [&](int v, int stg, int tj, uint32_t fb, uint32_t tx) {
            if (lane == 0) {
                if (tx > 0) mbar_expect_tx(fb, tx);
#pragma unroll
                for (int bx = 0; bx < C::NBOX; bx++)
                    tma_load_2d(sm_s + (v ? C::V_OFF : C::K_OFF) + (stg * C::NBOX + bx) * BOX, &tqkv, fb,
                                (nq + (v ? nk : 0) + kh) * HD + bx * 64, row0 + tj * BN);
            }
            __syncwarp();
        };
        // slots [a, b) of key tile `tile` from stage stg: (slot, box, K or V) items over the lanes
        auto store_slots = [&](int stg, int tile, int a, int b) {
            const int items = (b - a) * C::NBOX * 2;
            for (int it = lane; it < items; it += 32) {
                const int kv = it & 1, bx = (it >> 1) % C::NBOX, sl = a + (it >> 1) / C::NBOX;
                tma_store_3d(kv ? &tvc : &tkc, sm_s + (kv ? C::V_OFF : C::K_OFF) + (stg * C::NBOX + bx) * BOX,
                             bx * 64, tile * BN, sl * nk + kh);
            }
        };
        auto store_tile = [&](int stg, int tile) {
            store_slots(stg, tile, s0, s1);
            bulk_commit();
        };
        // planned: whether this CTA owns slot groups of key tile t (none past the plan's tiles)
        auto owns = [&](int t) {
            if (!planned || t < 0 || t >= PLAN_MAX || s0 >= s1) return false;
            for (int sg = 0; sg < PLAN_GROUPS; sg++)
                if (plan.owner[t][sg] == qt) return true;
            return false;
        };
        auto store_owned = [&](int stg, int t) {  // one bulk group per call
            for (int sg = 0; sg < PLAN_GROUPS; sg++) {
                const int a = s0 + sg * plan.gs, b = min(s1, a + plan.gs);
                if (plan.owner[t][sg] == qt && a < b) store_slots(stg, t, a, b);
            }
            bulk_commit();
        };
        // tile cj's K and V have both landed in stage cj & 1
        auto landed = [&](int t) {
            return __all_sync(0xffffffffu, mbar_wait(bar(B_KF0 + (t & 1)), (t >> 1) & 1) &&
                                               mbar_wait(bar(B_VF0 + (t & 1)), (t >> 1) & 1));
        };
        // planned epilogue, the key tiles from t0 on that this CTA owns groups of: loaded in turn into stages 0 and 1
        // (free: a copy CTA has no attention, and the others come here after the last use of both stages) and stored
        // from there; a stage is reloaded only once the stores of the tile two back have read it
        auto copy_planned = [&](int t0) {
            bool good = true;
            int i = 0;
            bulk_wait_read();  // the stores made during the attention have read their stages
            __syncwarp();
            for (int t = t0; t < ntiles_all && good; t++) {
                if (!owns(t)) continue;
                const int st = i & 1;
                const uint32_t cb = bar(st ? B_COPY1 : B_COPY);
                if (i >= 2) {  // every lane's stores of the tile two back have read the stage before lane 0 reloads it
                    bulk_wait_read_1();
                    __syncwarp();
                }
                load_half(0, st, t, cb, 2 * C::NBOX * BOX);
                load_half(1, st, t, cb, 0);
                good = __all_sync(0xffffffffu, *abort_flag == 0 && mbar_wait(cb, (i >> 1) & 1));
                if (good) store_owned(st, t);
                i++;
            }
            bulk_wait_read();  // shared memory stays in place until every store has read it
            return good;
        };
        bool ok = true, stored = false;
        if (copier) {
            ok = copy_planned(0);
            if (!ok && lane == 0) *abort_flag = 1;
            __syncwarp();
        } else {
            // The V loads trail the K loads by one tile (K0, K1, V0, K2, V1, ...): K_j waits only for S_{j-2}, never
            // behind the wait of a V stage for its P.V.
            for (int j = 0; j <= ntiles; j++) {
                if (j < ntiles) {
                    const int st = j & 1;
                    if (j >= 2) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_KE0 + st), ((j >> 1) - 1) & 1));
                    ok = __all_sync(0xffffffffu, ok && *abort_flag == 0);
                    if (!ok) break;
                    if ((copy && stored && j == cj + 2) || owns(j - 2)) {
                        // the stores of tile j - 2 (the latest bulk group) have read this stage, every lane's
                        bulk_wait_read();
                        __syncwarp();
                    }
                    load_half(0, st, j, bar(B_KF0 + st), C::NBOX * BOX);
                }
                if (j >= 1) {
                    const int v = j - 1, sv = v & 1;
                    if (v >= 2) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_VE0 + sv), ((v >> 1) - 1) & 1));
                    if (!ok) break;
                    load_half(1, sv, v, bar(B_VF0 + sv), C::NBOX * BOX);
                    if (copy && v == cj) {  // tile cj goes out as soon as both its halves have landed
                        ok = landed(cj);
                        if (!ok) break;
                        store_tile(cj & 1, cj);
                        stored = true;
                    }
                    if (owns(v)) {  // planned: this CTA's groups of tile v, as soon as it has landed
                        ok = landed(v);
                        if (!ok) break;
                        store_owned(v & 1, v);
                        stored = true;
                    }
                }
            }
            if (ok && copy && !stored) {
                if (cj < ntiles) {
                    // the CTA's last tile: still in its stage
                    ok = landed(cj);
                    if (ok) {
                        store_tile(cj & 1, cj);
                        stored = true;
                    }
                } else {
                    // a tile this CTA does not attend to: into stage 0 once its last use there (tile jl) is done
                    const int jl = (ntiles - 1) & ~1;
                    ok = __all_sync(0xffffffffu, mbar_wait(bar(B_KE0), (jl >> 1) & 1) &&
                                                     mbar_wait(bar(B_VE0), (jl >> 1) & 1));
                    if (ok) {
                        load_half(0, 0, cj, bar(B_COPY), 2 * C::NBOX * BOX);
                        load_half(1, 0, cj, bar(B_COPY), 0);
                        ok = __all_sync(0xffffffffu, mbar_wait(bar(B_COPY), 0));
                        if (ok) {
                            store_tile(0, cj);
                            stored = true;
                        }
                    }
                }
            }
            if (ok && planned) {
                // the last use of each stage (the last tile j of its parity: S read its K, P.V its V) must be done
                for (int st = 0; st < 2 && ok; st++) {
                    if (ntiles <= st) continue;
                    const int jl = ((ntiles - 1 - st) & ~1) + st;
                    ok = __all_sync(0xffffffffu, mbar_wait(bar(B_KE0 + st), (jl >> 1) & 1) &&
                                                     mbar_wait(bar(B_VE0 + st), (jl >> 1) & 1));
                }
                if (ok) ok = copy_planned(ntiles);
            }
            if (stored) bulk_wait_read();  // shared memory stays in place until every store has read it
            if (!ok && lane == 0) *abort_flag = 1;
            __syncwarp();  // the warp reaches the final CTA barrier converged
        }
    } else if (warp == 1 && !copier) {
        // ------------------------------ MMA issuer ------------------------------
        if (lane == 0) {
            const uint32_t idS = idesc_bf16_f32(BM, BN, 0, 0);
            const uint32_t idO = idesc_bf16_f32(BM, HD, 0, 1);
            const uint32_t tS = tmem, tO = tmem + C::O_COL;
            bool ok = mbar_wait(bar(B_Q), 0);
            auto issue_S = [&](int j) {
                const int st = j & 1;
                const uint32_t kbase = sm_s + C::K_OFF + st * C::NBOX * BOX;
#pragma unroll
                for (int ks = 0; ks < HD / 16; ks++) {
                    const uint64_t a = smem_desc_sw128(sm_s + C::Q_OFF + (ks >> 2) * BOX + (ks & 3) * 32, 16, 1024);
                    const uint64_t b = smem_desc_sw128(kbase + (ks >> 2) * BOX + (ks & 3) * 32, 16, 1024);
                    tc_mma_ss(tS, a, b, idS, ks > 0 ? 1u : 0u);
                }
                tc_commit(bar(B_SFULL));
                tc_commit(bar(B_KE0 + st));
            };
            if (ok && ntiles > 0) {
                ok = mbar_wait(bar(B_KF0), 0);
                if (ok) {
                    tc_fence_after();
                    issue_S(0);
                }
            }
            for (int j = 0; ok && j < ntiles; j++) {
                if (j + 1 < ntiles) {
                    // S_{j+1} may overwrite S_j once the softmax warps have read it
                    ok = mbar_wait(bar(B_KF0 + ((j + 1) & 1)), ((j + 1) >> 1) & 1) && mbar_wait(bar(B_SFREE), j & 1);
                    if (!ok) break;
                    tc_fence_after();
                    issue_S(j + 1);
                }
                ok = mbar_wait(bar(B_PFULL), j & 1) && mbar_wait(bar(B_VF0 + (j & 1)), (j >> 1) & 1);
                if (!ok) break;
                tc_fence_after();
                const uint32_t vbase = sm_s + C::V_OFF + (j & 1) * C::NBOX * BOX;
                const uint32_t tP = tmem + C::P_COL + (j & 1) * 128;  // hi at +0, lo at +64 (16 keys per 8 columns)
#pragma unroll
                for (int kk = 0; kk < BN / 16; kk++) {
                    const uint64_t b = smem_desc_sw128(vbase + kk * 2048, BOX, 1024);
                    tc_mma_ts(tO, tP + kk * 8, b, idO, (j > 0 || kk > 0) ? 1u : 0u);
                    tc_mma_ts(tO, tP + 64 + kk * 8, b, idO, 1u);
                }
                tc_commit(bar(B_ODONE));
                tc_commit(bar(B_PDONE0 + (j & 1)));
                tc_commit(bar(B_VE0 + (j & 1)));
            }
            if (!ok) *abort_flag = 1;
        }
        __syncwarp();
    } else if (!copier) {
        // ------------------------------ softmax / correction / epilogue ------------------------------
        const int quarter = warp & 3, wg = (warp - 2) >> 2;
        const int r = quarter * 32 + lane;  // query row within the tile
        const int qrow = q0 + r;            // position within the sequence
        const int cb = wg * 64;             // this warpgroup's columns [cb, cb + 64)
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        const uint32_t tS = tmem + lane_off, tO = tmem + lane_off + C::O_COL;
        constexpr int OH = HD / 2;          // O columns per warpgroup
        float m = -INFINITY, l = 0.f;       // max in log2 units of the scaled score; this thread's half of the sum
        bool ok = true;
        // Every softmax thread reaches the per-tile barrier in every iteration and the loop is left only on its
        // vote, so a wait that times out in one warp cannot leave the others at the barrier.
        for (int j = 0; j < ntiles; j++) {
            bool okt = ok && __all_sync(0xffffffffu, mbar_wait(bar(B_SFULL), j & 1));
            // keys [0, kmax) are visible; only the causal diagonal tile and a ragged last tile need the mask
            const int kbase = j * BN;
            const bool masked = (causal && kbase + BN - 1 > q0) || kbase + BN > seq;
            const int kmax = (causal ? min(seq, qrow + 1) : seq) - kbase;
            // this warpgroup's 64 columns of the row in one batch of loads; the row max meets its other half
            // through shared memory at the barrier
            uint32_t sr[64];
            float *mx = reinterpret_cast<float *>(sm + C::MX_OFF) + (j & 1) * 2 * BM;
            float mh = -INFINITY;
            if (okt) {
                tc_fence_after();
                tmem_ld32(tS + cb, sr);
                tmem_ld32(tS + cb + 32, sr + 32);
                tc_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(B_SFREE));
                if (masked) {  // CTA-uniform: only the causal diagonal tile and a ragged last tile
#pragma unroll
                    for (int c = 0; c < 64; c++)
                        if (cb + c >= kmax) sr[c] = __float_as_uint(-INFINITY);
                }
                float mt6[6];
#pragma unroll
                for (int k = 0; k < 6; k++) mt6[k] = -INFINITY;
#pragma unroll
                for (int c = 0; c < 60; c += 2)
                    mt6[(c >> 1) % 6] = fmax3(mt6[(c >> 1) % 6], __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
                mh = fmax3(fmax3(mt6[0], mt6[1], mt6[2]), fmax3(mt6[3], mt6[4], mt6[5]),
                           fmax3(__uint_as_float(sr[60]), __uint_as_float(sr[61]),
                                 fmaxf(__uint_as_float(sr[62]), __uint_as_float(sr[63]))));
                mx[wg * BM + r] = mh;
            }
            ok = bar_and<2, 256>(okt);
            if (!ok) break;
            const float mt = fmaxf(mh, mx[(1 - wg) * BM + r]) * sl2;
            // lazy rescaling: keep the stale max unless the new one exceeds it by more than 2^RESCALE_LOG2
            float alpha = 1.f;
            if (mt > m + RESCALE_LOG2) {
                alpha = fast_exp2(m - mt);  // 0 on the first tile (m = -inf)
                m = mt;
            }
            const float mref = m == -INFINITY ? 0.f : m;
            // P_j goes into buffer j & 1 once PV_{j-2} has read it (issued two tiles back, so this wait is short).
            // A wait that times out here ends the loop at the next tile's vote.
            if (j >= 2) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_PDONE0 + (j & 1)), ((j >> 1) - 1) & 1));
            if (!ok) continue;
            // p = 2^(s * sl2 - mref) per column, summed in eight independent chains (column c into chain c % 8), and
            // straight away this half of P row r (keys cb .. cb + 63) as bf16 pairs for TMEM buffer j & 1: hi (p
            // truncated to bf16, its upper 16 bits taken with a byte permute) in columns [32wg, 32wg + 32), lo (the
            // exact remainder p - hi rounded to bf16; hi + lo keeps ~16 bits of p) in [64 + 32wg, ...). One loop, so
            // the exponentials of a pair (multi-function unit) overlap the packing of the pairs before it (ALU); the
            // scaling, the sums and the remainders two columns per packed instruction. sr[k] takes the k-th hi pair
            // in place (pair k reads sr[2k], sr[2k + 1], which no earlier pair has written).
            float2 rs2[4];
#pragma unroll
            for (int k = 0; k < 4; k++) rs2[k] = make_float2(0.f, 0.f);
            const float2 sl2v = make_float2(sl2, sl2), nmref = make_float2(-mref, -mref);
            uint32_t lw[32];
#pragma unroll
            for (int i = 0; i < 32; i++) {
                const float2 x = fma2(make_float2(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1])), sl2v,
                                      nmref);
                // one pair in eight on the FMA pipe, the rest on the multi-function unit, which bounds this loop
                const float2 p = (i % 8) == 0 ? exp2_poly2(x) : make_float2(fast_exp2(x.x), fast_exp2(x.y));
                rs2[i & 3] = add2(rs2[i & 3], p);
                const uint32_t u0 = __float_as_uint(p.x), u1 = __float_as_uint(p.y);
                const float2 lo = sub2(p, make_float2(__uint_as_float(u0 & 0xffff0000u),
                                                      __uint_as_float(u1 & 0xffff0000u)));
                lw[i] = pack_bf16x2(lo.x, lo.y);
                sr[i] = __byte_perm(u0, u1, 0x7632);
            }
            const float rs = ((rs2[0].x + rs2[0].y) + (rs2[1].x + rs2[1].y)) +
                             ((rs2[2].x + rs2[2].y) + (rs2[3].x + rs2[3].y));
            l = l * alpha + rs;
            const uint32_t tPb = tmem + lane_off + C::P_COL + (j & 1) * 128;
            tmem_st32(tPb + wg * 32, sr);
            tmem_st32(tPb + 64 + wg * 32, lw);
            // O may be rescaled once PV_{j-1} has completed, and must be before PV_j starts (after PFULL)
            if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
                ok = __all_sync(0xffffffffu, mbar_wait(bar(B_ODONE), (j - 1) & 1));
                if (ok) {
                    tc_fence_after();
#pragma unroll
                    for (int c = 0; c < OH; c += 32) {
                        uint32_t orow[32];
                        tmem_ld32(tO + wg * OH + c, orow);
                        tc_wait_ld();
#pragma unroll
                        for (int k = 0; k < 32; k++) orow[k] = __float_as_uint(__uint_as_float(orow[k]) * alpha);
                        tmem_st32(tO + wg * OH + c, orow);
                    }
                }
            }
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (!ok) continue;
            if (lane == 0) mbar_arrive(bar(B_PFULL));
        }
        // O is final once the last P.V has completed: waited on that P buffer's barrier, whose phase before it (the
        // P.V two tiles back) this loop has already waited for, so the parity names one phase only. (B_ODONE could
        // still be two phases behind here, where a parity wait cannot tell the phase awaited from the one before.)
        if (ok && ntiles > 0)
            ok = __all_sync(0xffffffffu,
                            mbar_wait(bar(B_PDONE0 + ((ntiles - 1) & 1)), ((ntiles - 1) >> 1) & 1));
        if (!ok) *abort_flag = 1;
        // the two halves of each row sum meet in shared memory
        float *lx = reinterpret_cast<float *>(sm + C::LX_OFF);
        lx[wg * BM + r] = l;
        asm volatile("bar.sync 1, 256;" ::: "memory");
        const float ltot = l + lx[(1 - wg) * BM + r];
        if (ok && ntiles > 0) {
            tc_fence_after();
            const float inv = 1.f / ltot;
            bf16 *dst = out + static_cast<long>(row0 + qrow) * nq * HD + h * HD + wg * OH;
#pragma unroll
            for (int c = 0; c < OH; c += 32) {
                uint32_t orow[32];
                tmem_ld32(tO + wg * OH + c, orow);
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
    if (warp == 1 && !copier) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

}  // namespace pf
