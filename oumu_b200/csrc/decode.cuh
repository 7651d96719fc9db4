// Split-KV GQA decode attention for sm_100a with the cross-split combine fused in, optionally with the decode
// prologue (rope of q and k at the newest position, k/v written into the take's cache slot) fused in as well.
//
// Work unit: a tile of 32 KV positions of one (take, kv head) "segment". All tiles of all segments are laid end to
// end (take-major, then kv head, then position) and cut into equal contiguous ranges, one per CTA, so every CTA
// streams the same number of bytes whatever the per-take lengths are. A segment entirely inside one CTA is
// finished there; a segment split across CTAs leaves one partial per CTA and the last CTA to finish (atomic
// counter, no waiting) merges them.
//
// Warp roles per CTA:
//   warps 0..5  consumers: tile i of the CTA's range -> warp i % 6 and stage i % 12 (two stages per warp, one
//               computing while the other loads), each warp with its own online-softmax state. Per tile, for the
//               two 16-position halves (independent mma chains):
//                 S^T[16 pos x 8 heads] = K[16 x hd] . Q^T[hd x 8]   (mma.sync m16n8k16; A = K via ldmatrix,
//                                                                     B = q in registers)
//                 online softmax down the position axis (fp32, exp2 with the scale folded)
//                 O^T[hd x 8 heads] += V^T[hd x 16] . P^T[16 x 8]    (A = V via ldmatrix.trans, B = P via
//                                                                     movmatrix, P as bf16 hi + lo ~ 16 bits)
//               At a segment end each warp drops its state into a shared-memory slot and goes on; the CTA's last
//               segment end is merged by the consumer warps together.
//   warp 6      producer: streams K and V tiles with TMA (128-byte swizzle) into the stages, in order.
//               Fused form: the consumer warp that owns a segment's last tile rotates the newest position's k
//               (rope), writes k and v into the cache slot and patches them into the shared-memory tile.
//   warp 7      merger: merges the consumer warp states of each earlier segment end, writes the output (or the CTA's
//               partial, and merges all CTAs' partials when it is the last contributor), off the streaming path.
// Each KV byte is read from HBM once for all q heads of its GQA group (the reference reads it once per q head,
// kernels/voxcpm.cu:139-148).
// With programmatic dependent launch (oumu_set_pdl) the set-up and the loads of cache tiles that the preceding
// kernel cannot be writing (every tile below the newest position) overlap the preceding kernel; q, the tile that
// holds the newest position, and every global write wait for it (griddepcontrol.wait).
#pragma once
#include "common.cuh"

namespace dec {

constexpr int TILE = 32;     // KV positions per stage
constexpr int NCW = 6;       // consumer warps
constexpr int PRODUCER = NCW, MERGER = NCW + 1;
constexpr int NTHREADS = (NCW + 2) * 32;
constexpr int GMAX = 8;      // q heads per kv head handled by one mma column block
// Two stages per consumer warp: tile i of a CTA's range goes to warp i % NCW and stage i % STAGES, so stage s is
// only ever read by warp s % NCW, which waits on its phases strictly in order while its other stage loads. (A warp
// that could reach a stage's phase two ahead of the barrier would be misled: mbarrier parity waits cannot tell it
// from the phase before.)
constexpr int STAGES = 2 * NCW;
constexpr int NFB = 1;       // flush buffer between the consumers and the merger
constexpr int MIN_TILES = 4; // tiles per CTA at least: small problems use fewer CTAs rather than many 1-tile partials
// ... and no segment split over more than about MAX_SPLIT CTAs, with ranges of up to SPLIT_TILES_MAX tiles: a split
// segment's last contributor merges every partial in turn, so one long take decoded alone is better served by a few
// CTAs with more tiles each (one take of 4096 positions: 23.7 -> 14.7 us; of 16384: 44.3 -> 31.4 us)
constexpr int MAX_SPLIT = 8, SPLIT_TILES_MAX = 64;

template <int HD>
struct Cfg {
    static constexpr int NBOX = HD / 64;                   // 64-element (128-byte) TMA boxes per row
    static constexpr int BOX_BYTES = TILE * 128;           // 32 rows x 128 B
    static constexpr int KV_BYTES = NBOX * BOX_BYTES;      // one K (or V) tile
    static constexpr int STAGE_BYTES = 2 * KV_BYTES;
    static constexpr int PART_FLOATS = 2 * GMAX + GMAX * HD;  // m[8], l[8], o[8][HD]
    static constexpr int FLUSH_BYTES = NFB * NCW * PART_FLOATS * 4;
};

struct Params {
    bf16 *qkv;            // read; the fused form also writes the rotated k of the newest position back
    bf16 *kc, *vc;        // caches (written only by the fused form, at the newest position)
    bf16 *out;
    float *part;          // [gridDim.x][2][PART_FLOATS]
    int *cnt;             // [B * nk], zero between launches
    const int *pos;
    const int *lens;
    const float *cos_t, *sin_t;  // fused form: rotary tables, or null (no rope)
    int B, nq, nk, maxlen;
    float sl2;            // scale * log2(e)
};

// Shared-memory layout (offsets from the 1024-aligned base).
template <int HD>
struct Smem {
    int B;
    __host__ __device__ int flush_off() const { return STAGES * Cfg<HD>::STAGE_BYTES; }
    __host__ __device__ int bar_off() const { return flush_off() + Cfg<HD>::FLUSH_BYTES; }
    __host__ __device__ int pre_off() const { return bar_off() + (2 * STAGES + 2 * NFB) * 8; }
    __host__ __device__ int len_off() const { return pre_off() + (B + 1) * 4; }
    __host__ __device__ int misc_off() const { return len_off() + B * 4; }
    __host__ __device__ int bytes() const { return misc_off() + 16; }
};

// Iterator over the tiles of the segments: segment (s, kh), tile j of T = ceil(L / TILE).
struct TileIt {
    int s, kh, j, T, L;
    __device__ void seek(long t, const int *pre, const int *Ls, int B) {
        int lo = 0, hi = B - 1;
        while (lo < hi) {  // largest s with pre[s] <= t
            int mid = (lo + hi + 1) >> 1;
            if (pre[mid] <= t) lo = mid; else hi = mid - 1;
        }
        s = lo;
        L = Ls[s];
        T = (L + TILE - 1) / TILE;
        int off = static_cast<int>(t - pre[s]);
        kh = off / T;
        j = off % T;
    }
    __device__ void next(const int *Ls, int nk) {
        if (++j == T) {
            j = 0;
            if (++kh == nk) {
                kh = 0;
                ++s;
                L = Ls[s];
                T = (L + TILE - 1) / TILE;
            }
        }
    }
};

__device__ __forceinline__ void bar_consumers() { asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory"); }
// End of the CTA's streaming: the consumer warps arrive (without waiting), the producer warp waits for them.
__device__ __forceinline__ void bar_end_arrive() { asm volatile("bar.arrive 2, %0;" ::"n"((NCW + 1) * 32) : "memory"); }
__device__ __forceinline__ void bar_end_sync() { asm volatile("bar.sync 2, %0;" ::"n"((NCW + 1) * 32) : "memory"); }

// CTA whose tile range contains tile t (ranges [c*W/G, (c+1)*W/G)).
__device__ __forceinline__ int cta_of(long t, long W, int G) {
    return static_cast<int>(((t + 1) * G + W - 1) / W) - 1;
}

// Merge of one segment end, run by NT threads (32: the merger warp; NCW*32: the consumer warps together).
// Thread i owns hd columns [lane*DL, lane*DL + DL) of heads i/32 + k*NT/32, so shared-memory reads, partial records
// and outputs are contiguous across each warp. F holds the NCW warp states (m[8], l[8], o[8][HD] each); `release`
// runs as soon as they are read (the merger hands the flush buffer back to the consumers there, before its global
// writes and the cross-CTA round trips). Writes the segment's output when the whole segment is in this CTA;
// otherwise this CTA's partial, and if it is the last contributor (atomic counter) merges every contributor's
// partial and writes the output. At the CTA's last segment end, a CTA that finds every other contributor already
// published is the last one and merges with its own partial still in registers, publishing nothing.
template <int HD, int NT, class Release>
__device__ __forceinline__ void merge_segment(const Params &P, const float *F, int s, int kh, long Sg, long Eg,
                                              long ta, long tb, long W, int Gc, int c, int slot, int tid,
                                              volatile int *bcast, Release release) {
    using C = Cfg<HD>;
    constexpr int DL = HD / 32;         // hd columns per thread: 4 (hd 128) or 2 (hd 64)
    constexpr int HS = NT / 32;                 // head stride between a thread's heads
    constexpr int NH = (GMAX + HS - 1) / HS;    // heads per thread (the last may be past GMAX)
    auto sync = [] {
        if constexpr (NT == 32) __syncwarp(); else bar_consumers();
    };
    const int G = P.nq / P.nk, g = s * P.nk + kh;
    const int lane = tid & 31, hb = tid >> 5, d0 = lane * DL;
    const bool whole = Sg >= ta && Eg <= tb;
    float Mx[NH], Lsum[NH], o[NH][DL];
#pragma unroll
    for (int k = 0; k < NH; k++) {
        Mx[k] = -INFINITY;
        Lsum[k] = 0.f;
#pragma unroll
        for (int e = 0; e < DL; e++) o[k][e] = 0.f;
    }
#pragma unroll
    for (int w = 0; w < NCW; w++)
#pragma unroll
        for (int k = 0; k < NH; k++)
            if (hb + k * HS < GMAX) Mx[k] = fmaxf(Mx[k], F[w * C::PART_FLOATS + hb + k * HS]);
#pragma unroll
    for (int w = 0; w < NCW; w++) {
        const float *Fw = F + w * C::PART_FLOATS;
#pragma unroll
        for (int k = 0; k < NH; k++) {
            const int h = hb + k * HS;
            if (h >= GMAX) continue;
            const float mw = Fw[h];
            const float cw = mw == -INFINITY ? 0.f : fast_exp2(mw - Mx[k]);
            Lsum[k] += cw * Fw[GMAX + h];
            const float *ow = Fw + 2 * GMAX + h * HD + d0;
            if constexpr (DL == 4) {
                const float4 u = *reinterpret_cast<const float4 *>(ow);
                o[k][0] += cw * u.x; o[k][1] += cw * u.y; o[k][2] += cw * u.z; o[k][3] += cw * u.w;
            } else {
                const float2 u = *reinterpret_cast<const float2 *>(ow);
                o[k][0] += cw * u.x; o[k][1] += cw * u.y;
            }
        }
    }
    release();
    bf16 *dst = P.out + static_cast<long>(s) * P.nq * HD + kh * G * HD + d0;
    auto store = [&](const float (&l)[NH]) {
#pragma unroll
        for (int k = 0; k < NH; k++) {
            const int h = hb + k * HS;
            if (h < G && h < GMAX) {
                if constexpr (DL == 4) {
                    uint2 u;
                    u.x = pack_bf16x2(o[k][0] / l[k], o[k][1] / l[k]);
                    u.y = pack_bf16x2(o[k][2] / l[k], o[k][3] / l[k]);
                    *reinterpret_cast<uint2 *>(dst + h * HD) = u;
                } else {
                    *reinterpret_cast<uint32_t *>(dst + h * HD) = pack_bf16x2(o[k][0] / l[k], o[k][1] / l[k]);
                }
            }
        }
    };
    if (whole) {
        store(Lsum);
        return;
    }
    const int cf = cta_of(Sg, W, Gc), cl = cta_of(Eg - 1, W, Gc);
    // At the CTA's last segment end (the consumer warps' merge): when every other contributor has already published
    // (the usual case: the next CTA streamed its part of this segment first), this CTA is the last one and merges
    // without publishing its own partial. The merge warp's partials are CTAs' first segments, whose other
    // contributors finish later, so it publishes directly without the extra round trip.
    bool own_in_regs = false;
    if constexpr (NT != 32) {
        if (tid == 0) *bcast = ld_acquire_gpu(P.cnt + g);
        sync();
        own_in_regs = *bcast == cl - cf;
        sync();
    }
    if (!own_in_regs) {
        float *rec = P.part + (static_cast<long>(c) * 2 + slot) * C::PART_FLOATS;
        if (lane == 0) {
#pragma unroll
            for (int k = 0; k < NH; k++) {
                if (hb + k * HS >= GMAX) continue;
                rec[hb + k * HS] = Mx[k];
                rec[GMAX + hb + k * HS] = Lsum[k];
            }
        }
#pragma unroll
        for (int k = 0; k < NH; k++) {
            if (hb + k * HS >= GMAX) continue;
            float *ro = rec + 2 * GMAX + (hb + k * HS) * HD + d0;
            if constexpr (DL == 4) *reinterpret_cast<float4 *>(ro) = make_float4(o[k][0], o[k][1], o[k][2], o[k][3]);
            else *reinterpret_cast<float2 *>(ro) = make_float2(o[k][0], o[k][1]);
        }
        // publish: the threads' writes are ordered before thread 0's release by the barrier; the acquire side of
        // the same atomic orders the last contributor's reads of the other partials after their writers' releases
        sync();
        if (tid == 0) *bcast = atomic_add_acq_rel(P.cnt + g, 1);
        sync();
        const int old = *bcast;
        sync();
        if (old != cl - cf) return;
    }
    // last contributor: merge every CTA's partial of this segment in one online pass, in CTA order (this CTA's own
    // from registers or from its record: the same values and the same arithmetic either way; the records of four
    // contributors are loaded together: one round trip to L2 per four)
    float Mo[NH], Lo[NH], oo[NH][DL];
#pragma unroll
    for (int k = 0; k < NH; k++) {
        Mo[k] = Mx[k];
        Lo[k] = Lsum[k];
#pragma unroll
        for (int e = 0; e < DL; e++) oo[k][e] = o[k][e];
    }
    float M2[NH], L2[NH];
#pragma unroll
    for (int k = 0; k < NH; k++) {
        M2[k] = -INFINITY;
        L2[k] = 0.f;
#pragma unroll
        for (int e = 0; e < DL; e++) o[k][e] = 0.f;
    }
#pragma unroll 4
    for (int cc = cf; cc <= cl; cc++) {
        const long ac = static_cast<long>(cc) * W / Gc;
        const float *rc = P.part + (static_cast<long>(cc) * 2 + ((cc == cf && ac < Sg) ? 1 : 0)) * C::PART_FLOATS;
        float mc[NH], lc[NH], oc[NH][DL];
        const bool own = own_in_regs && cc == c;
#pragma unroll
        for (int k = 0; k < NH; k++) {
            if (own) {
                mc[k] = Mo[k];
                lc[k] = Lo[k];
#pragma unroll
                for (int e = 0; e < DL; e++) oc[k][e] = oo[k][e];
                continue;
            }
            const int h = hb + k * HS < GMAX ? hb + k * HS : 0;
            mc[k] = __ldcg(rc + h);
            lc[k] = __ldcg(rc + GMAX + h);
            const float *op = rc + 2 * GMAX + h * HD + d0;
            if constexpr (DL == 4) {
                const float4 u = __ldcg(reinterpret_cast<const float4 *>(op));
                oc[k][0] = u.x; oc[k][1] = u.y; oc[k][2] = u.z; oc[k][3] = u.w;
            } else {
                const float2 u = __ldcg(reinterpret_cast<const float2 *>(op));
                oc[k][0] = u.x; oc[k][1] = u.y;
            }
        }
#pragma unroll
        for (int k = 0; k < NH; k++) {
            if (hb + k * HS >= GMAX || mc[k] == -INFINITY) continue;
            const float mn = fmaxf(M2[k], mc[k]);
            const float wa = M2[k] == -INFINITY ? 0.f : fast_exp2(M2[k] - mn);
            const float wc = fast_exp2(mc[k] - mn);
            M2[k] = mn;
            L2[k] = L2[k] * wa + lc[k] * wc;
#pragma unroll
            for (int e = 0; e < DL; e++) o[k][e] = o[k][e] * wa + oc[k][e] * wc;
        }
    }
    store(L2);
    if (tid == 0) P.cnt[g] = 0;
}

// Fused form: the newest position's k and v, handled by the consumer warp that owns the segment's last tile.
// newest_load fetches the raw rows (lanes < KG: 8 rope pairs of k each, with their rotary table entries; the next
// VC lanes: 16 bytes of v each), all before the tile is awaited; newest_store rotates k (same arithmetic as the
// rope kernel, kernels/voxcpm.cu:109-114), writes k and v into the cache slot and the rotated k back into qkv (in
// place, like rope), and patches row r of the shared-memory tile that TMA loaded before the position was written.
template <int HD>
struct Newest {
    static constexpr int HALF = HD / 2, KG = HALF / 8, VC = HD / 8;
    uint4 a, b;
    float4 c0, c1, s0, s1;
    __device__ __forceinline__ void load(const Params &P, int s, int kh, int p, int lane) {
        const bf16 *row = P.qkv + static_cast<long>(s) * (P.nq + 2 * P.nk) * HD;
        if (lane < KG) {
            const bf16 *k = row + (P.nq + kh) * HD + lane * 8;
            a = *reinterpret_cast<const uint4 *>(k);
            b = *reinterpret_cast<const uint4 *>(k + HALF);
            if (P.cos_t) {
                const float4 *cp = reinterpret_cast<const float4 *>(P.cos_t + static_cast<long>(p) * HALF + lane * 8);
                const float4 *sp = reinterpret_cast<const float4 *>(P.sin_t + static_cast<long>(p) * HALF + lane * 8);
                c0 = cp[0];
                c1 = cp[1];
                s0 = sp[0];
                s1 = sp[1];
            }
        } else if (lane < KG + VC) {
            a = reinterpret_cast<const uint4 *>(row + (P.nq + P.nk + kh) * HD)[lane - KG];
        }
    }
    __device__ __forceinline__ void store(const Params &P, int s, int kh, int p, int lane, uint32_t kb, uint32_t vb,
                                          int r) {
        const long dst = ((static_cast<long>(s) * P.nk + kh) * P.maxlen + p) * HD;
        if (lane < KG) {
            const int i = lane * 8;
            if (P.cos_t) {
                const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
                const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
                const bf16 *x = reinterpret_cast<const bf16 *>(&a);
                const bf16 *y = reinterpret_cast<const bf16 *>(&b);
                uint4 o1, o2;
                bf16 *oa = reinterpret_cast<bf16 *>(&o1);
                bf16 *ob = reinterpret_cast<bf16 *>(&o2);
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    const float x1 = bf2f(x[e]), x2 = bf2f(y[e]);
                    oa[e] = f2bf(x1 * cs[e] - x2 * sn[e]);
                    ob[e] = f2bf(x2 * cs[e] + x1 * sn[e]);
                }
                a = o1;
                b = o2;
                bf16 *k = P.qkv + static_cast<long>(s) * (P.nq + 2 * P.nk) * HD + (P.nq + kh) * HD + i;
                *reinterpret_cast<uint4 *>(k) = a;
                *reinterpret_cast<uint4 *>(k + HALF) = b;
            }
            *reinterpret_cast<uint4 *>(P.kc + dst + i) = a;
            *reinterpret_cast<uint4 *>(P.kc + dst + i + HALF) = b;
            const int c1 = i / 8, c2 = (i + HALF) / 8;  // 16-byte chunk index within the row
            st_shared_v4(kb + (c1 >> 3) * Cfg<HD>::BOX_BYTES + sw128(r, c1 & 7), a);
            st_shared_v4(kb + (c2 >> 3) * Cfg<HD>::BOX_BYTES + sw128(r, c2 & 7), b);
        } else if (lane < KG + VC) {
            const int ch = lane - KG;
            reinterpret_cast<uint4 *>(P.vc + dst)[ch] = a;
            st_shared_v4(vb + (ch >> 3) * Cfg<HD>::BOX_BYTES + sw128(r, ch & 7), a);
        }
    }
};

// Fused form, consumers: rotate the q fragments (B operand: qb[ks][0] = q[16ks + c2, +1], qb[ks][1] = +8) at
// position p. Element d pairs with d + HD/2, which this lane holds in fragment ks + HD/32.
template <int HD>
__device__ __forceinline__ void rope_q_frags(uint32_t (&qb)[HD / 16][2], const float *cos_t, const float *sin_t,
                                             int p, int c2) {
    constexpr int HALF = HD / 2, H = HD / 32;
    const float *cr = cos_t + static_cast<long>(p) * HALF, *sr = sin_t + static_cast<long>(p) * HALF;
#pragma unroll
    for (int ks = 0; ks < H; ks++) {
#pragma unroll
        for (int f = 0; f < 2; f++) {
            const int d = ks * 16 + f * 8 + c2;
            const float2 cc = *reinterpret_cast<const float2 *>(cr + d);
            const float2 ss = *reinterpret_cast<const float2 *>(sr + d);
            const float2 x1 = unpack_bf16x2(qb[ks][f]), x2 = unpack_bf16x2(qb[ks + H][f]);
            qb[ks][f] = pack_bf16x2(x1.x * cc.x - x2.x * ss.x, x1.y * cc.y - x2.y * ss.y);
            qb[ks + H][f] = pack_bf16x2(x2.x * cc.x + x1.x * ss.x, x2.y * cc.y + x1.y * ss.y);
        }
    }
}

// DROP: the fault-injection build used by the failure-detection tests (oumu_test_drop_last_tile): CTA 0 never loads
// the last tile of its range, so the consumer that owns it waits until the limit; the producer then lets every copy
// it issued land before the CTA exits. Everything else is the same code.
template <int HD, bool FUSED, bool DROP = false>
__global__ void __launch_bounds__(NTHREADS, 1)
    k_attn_decode(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv, Params P) {
    using C = Cfg<HD>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_s = smem_u32(smem_raw);
    uint8_t *sm = smem_raw + ((1024u - (raw_s & 1023u)) & 1023u);
    const uint32_t sm_s = smem_u32(sm);
    const Smem<HD> L{P.B};
    float *flush = reinterpret_cast<float *>(sm + L.flush_off());
    const uint32_t bar_full = sm_s + L.bar_off();
    const uint32_t bar_empty = bar_full + 8 * STAGES;
    const uint32_t bar_ffull = bar_empty + 8 * STAGES;  // flush buffer b written by all consumer warps
    const uint32_t bar_fempty = bar_ffull + 8 * NFB;    // flush buffer b merged, free again
    int *pre = reinterpret_cast<int *>(sm + L.pre_off());
    int *Ls = reinterpret_cast<int *>(sm + L.len_off());
    volatile int *misc = reinterpret_cast<volatile int *>(sm + L.misc_off());  // [abort, bcast, bcast, longest]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int B = P.B, nk = P.nk, G = P.nq / P.nk;

    // the tensor maps' descriptors are fetched while warp 0 scans the lengths
    if (threadIdx.x == PRODUCER * 32) {
        tma_prefetch_desc(&tk);
        tma_prefetch_desc(&tv);
    }
    // ---- per-take lengths and the tile prefix over takes (warp 0) ----
    if (warp == 0) {
        const int per = (B + 31) / 32, s0 = lane * per;
        int sum = 0, tmax = 0;
        for (int k = 0; k < per; k++) {
            int s = s0 + k;
            if (s < B) {
                int Lv = P.lens ? P.lens[s] : *P.pos + 1;
                if (Lv < 1 || Lv > P.maxlen) {
                    record_error(OUMU_DEVERR_LENGTH);
                    Lv = Lv < 1 ? 1 : P.maxlen;
                }
                Ls[s] = Lv;
                const int T = (Lv + TILE - 1) / TILE;
                sum += T * nk;
                tmax = T > tmax ? T : tmax;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) tmax = max(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
        if (lane == 0) misc[3] = tmax;  // the longest segment, in tiles
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int run = incl - sum;
        for (int k = 0; k < per; k++) {
            int s = s0 + k;
            if (s < B) {
                pre[s] = run;
                run += ((Ls[s] + TILE - 1) / TILE) * nk;
            }
        }
        if (lane == 31) pre[B] = incl;
    } else if (threadIdx.x == 32) {
        for (int i = 0; i < STAGES; i++) {
            mbar_init(bar_full + 8 * i, 1);
            mbar_init(bar_empty + 8 * i, 1);
        }
        for (int b = 0; b < NFB; b++) {
            mbar_init(bar_ffull + 8 * b, NCW);
            mbar_init(bar_fempty + 8 * b, 1);
        }
        misc[0] = 0;  // abort flag
        mbar_fence_init();
    }
    __syncthreads();

    // Effective grid: at most one CTA per MIN_TILES tiles, so every CTA range [c*W/Gc, (c+1)*W/Gc) is non-empty and
    // every CTA between the first and the last of a segment contributes a partial to it; and fewer, longer ranges when
    // the longest segment would otherwise be split over more than about MAX_SPLIT CTAs.
    const long W = pre[B];
    const int split_tiles = min((misc[3] + MAX_SPLIT - 1) / MAX_SPLIT, SPLIT_TILES_MAX);
    const long min_tiles = split_tiles > MIN_TILES ? split_tiles : MIN_TILES;
    const long want = (W + min_tiles - 1) / min_tiles;
    const int Gc = static_cast<int>(want < static_cast<long>(gridDim.x) ? want : static_cast<long>(gridDim.x));
    const int c = blockIdx.x;
    if (threadIdx.x == 0) pdl_trigger();
    if (c >= Gc) return;
    const long ta = static_cast<long>(c) * W / Gc, tb = static_cast<long>(c + 1) * W / Gc;

    if (warp == PRODUCER) {
        // ------------------------------ producer ------------------------------
        int st = 0;
        uint32_t use = 0;
        if (lane == 0) {
            TileIt it;
            it.seek(ta, pre, Ls, B);
            const long tend = DROP && c == 0 ? tb - 1 : tb;
            // the unfused form reads the newest position only after the kernel that wrote it (the prologue)
            bool waited = FUSED;
            for (long t = ta; t < tend; t++) {
                if (!waited && it.j == it.T - 1) {
                    pdl_wait();
                    waited = true;
                }
                if (use > 0 && !mbar_wait(bar_empty + 8 * st, (use - 1) & 1u)) {
                    misc[0] = 1;
                    break;
                }
                if (misc[0]) break;
                const uint32_t fb = bar_full + 8 * st;
                mbar_expect_tx(fb, C::STAGE_BYTES);
                const int row = (it.s * nk + it.kh) * P.maxlen + it.j * TILE;
                const uint32_t kdst = sm_s + st * C::STAGE_BYTES;
#pragma unroll
                for (int bx = 0; bx < C::NBOX; bx++) {
                    tma_load_2d(kdst + bx * C::BOX_BYTES, &tk, fb, bx * 64, row);
                    tma_load_2d(kdst + C::KV_BYTES + bx * C::BOX_BYTES, &tv, fb, bx * 64, row);
                }
                if (t + 1 < tb) it.next(Ls, nk);
                if (++st == STAGES) {
                    st = 0;
                    ++use;
                }
            }
        }
        // DROP build: once every consumer warp is done (a hardware barrier: the warp sleeps, no polling), after an
        // abort (the consumers no longer wait for their tiles) this thread waits, bounded, until every load it
        // issued has landed, since a copy must not write shared memory of a CTA that has left. Stage s's last load
        // is of phase `use` if s < st, else of `use - 1` (none if use == 0). In the normal build the consumers have
        // waited for every load.
        if constexpr (DROP) {
            __syncwarp();
            bar_end_sync();
            if (lane == 0 && misc[0]) {
                for (int s2 = 0; s2 < STAGES; s2++) {
                    if (s2 >= st && use == 0) continue;
                    const uint32_t ph = s2 < st ? use : use - 1;
                    mbar_wait(bar_full + 8 * s2, ph & 1u);
                }
            }
        }
        return;
    }

    if (warp == MERGER) {
        // ------------------------------ merger: every segment end but the CTA's last ------------------------------
        TileIt it;
        it.seek(ta, pre, Ls, B);
        int nflush = 0;
        pdl_wait();  // global writes only after the preceding kernel
        for (long t = ta; t < tb - 1; t++) {
            if (it.j == it.T - 1) {
                const int b = nflush % NFB;
                // after an abort (a wait that ran out anywhere in the CTA) nothing is waited for any more, but every
                // merge still runs, on whatever the buffers hold: each contributor of a split segment still counts
                // itself, so the segment's last contributor resets the counter and the workspace stays usable
                const bool ok = __all_sync(0xffffffffu, misc[0] == 0 &&
                                                            mbar_wait(bar_ffull + 8 * b, (nflush / NFB) & 1));
                if (!ok) misc[0] = 1;
                const long Sg = pre[it.s] + static_cast<long>(it.kh) * it.T;
                merge_segment<HD, 32>(P, flush + b * NCW * C::PART_FLOATS, it.s, it.kh, Sg, Sg + it.T, ta, tb, W,
                                      Gc, c, nflush == 0 ? 0 : 1, lane, misc + 2, [&] {
                                          __syncwarp();
                                          if (lane == 0) mbar_arrive(bar_fempty + 8 * b);
                                      });
                __syncwarp();
                nflush++;
            }
            it.next(Ls, nk);
        }
        return;
    }

    // ------------------------------ consumers ------------------------------
    const int r4 = lane >> 2, c2 = (lane & 3) * 2, mi = lane >> 3;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float acc[HD / 16][4];
#pragma unroll
    for (int mt = 0; mt < HD / 16; mt++) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
    uint32_t qb[HD / 16][2];
    bool need_q = true;
    int nflush = 0;

    TileIt it;
    it.seek(ta, pre, Ls, B);
    if (ta + warp < tb) {
        // L2 prefetch of the q rows (and rotary-table rows) of this warp's first segment before the wait, so the q
        // load after it finds them in L2. A hint only: q written by the preceding kernel is still read correctly.
        TileIt f = it;
        for (int k = 0; k < warp; k++) f.next(Ls, nk);
        const char *q = reinterpret_cast<const char *>(P.qkv + static_cast<long>(f.s) * (P.nq + 2 * nk) * HD +
                                                       f.kh * G * HD);
        if (lane * 128 < G * HD * 2) prefetch_l2(q + lane * 128);
        if (FUSED && P.cos_t && lane < 2 * (HD * 2 / 128)) {
            const float *tab = lane < HD * 2 / 128 ? P.cos_t : P.sin_t;
            prefetch_l2(tab + static_cast<long>(f.L - 1) * (HD / 2) + (lane % (HD * 2 / 128)) * 32);
        }
    }
    pdl_wait();           // q is written upstream
    int owner = 0;
    uint32_t ntile = 0;   // tiles this warp has taken: its k-th tile is in stage warp + (k & 1) * NCW
    for (long t = ta; t < tb; t++) {
        if (owner == warp) {
            if (need_q) {
                const bf16 *q = P.qkv + static_cast<long>(it.s) * (P.nq + 2 * nk) * HD + (it.kh * G + r4) * HD;
#pragma unroll
                for (int ks = 0; ks < HD / 16; ks++) {
                    if (r4 < G) {
                        qb[ks][0] = *reinterpret_cast<const uint32_t *>(q + ks * 16 + c2);
                        qb[ks][1] = *reinterpret_cast<const uint32_t *>(q + ks * 16 + 8 + c2);
                    } else {
                        qb[ks][0] = qb[ks][1] = 0u;
                    }
                }
                if (FUSED && P.cos_t && r4 < G) rope_q_frags<HD>(qb, P.cos_t, P.sin_t, it.L - 1, c2);
                need_q = false;
            }
            const int st = warp + static_cast<int>(ntile & 1u) * NCW;
            const uint32_t use = ntile >> 1;
            const bool newest = FUSED && it.j == it.T - 1;
            Newest<HD> nw;
            if (newest) nw.load(P, it.s, it.kh, it.L - 1, lane);  // in flight while the tile is awaited
            bool ok = misc[0] == 0;
            if (ok && !mbar_wait(bar_full + 8 * st, use & 1u)) {
                misc[0] = 1;
                ok = false;
            }
            ok = __all_sync(0xffffffffu, ok);
            const int p0 = it.j * TILE;
            if (ok) {
                const uint32_t kb = sm_s + st * C::STAGE_BYTES, vb = kb + C::KV_BYTES;
                if (newest) {
                    nw.store(P, it.s, it.kh, it.L - 1, lane, kb, vb, it.L - 1 - p0);
                    __syncwarp();
                }
                // S^T for the two 16-position halves (independent chains)
                float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
                for (int ks = 0; ks < HD / 16; ks++) {
#pragma unroll
                    for (int h2 = 0; h2 < 2; h2++) {
                        uint32_t a0, a1, a2, a3;
                        const int krow = h2 * 16 + (mi & 1) * 8 + (lane & 7);
                        ldsm_x4(kb + (ks >> 2) * C::BOX_BYTES + sw128(krow, 2 * (ks & 3) + (mi >> 1)), a0, a1, a2,
                                a3);
                        mma_bf16_16816(s[h2], a0, a1, a2, a3, qb[ks][0], qb[ks][1]);
                    }
                }
                float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
                for (int h2 = 0; h2 < 2; h2++) {
                    const int pr0 = p0 + h2 * 16 + r4;
#pragma unroll
                    for (int k = 0; k < 4; k++) s[h2][k] *= P.sl2;
                    if (pr0 >= it.L) s[h2][0] = s[h2][1] = -INFINITY;
                    if (pr0 + 8 >= it.L) s[h2][2] = s[h2][3] = -INFINITY;
                    mx0 = fmaxf(mx0, fmaxf(s[h2][0], s[h2][2]));
                    mx1 = fmaxf(mx1, fmaxf(s[h2][1], s[h2][3]));
                }
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) {
                    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
                    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
                }
                // position p0 < L always, so the tile maxima are finite
                const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
                const float al0 = fast_exp2(m0 - mn0), al1 = fast_exp2(m1 - mn1);
                m0 = mn0;
                m1 = mn1;
                uint32_t ph[2][2], pl[2][2];
#pragma unroll
                for (int h2 = 0; h2 < 2; h2++) {
                    const float p00 = fast_exp2(s[h2][0] - mn0), p01 = fast_exp2(s[h2][1] - mn1);
                    const float p10 = fast_exp2(s[h2][2] - mn0), p11 = fast_exp2(s[h2][3] - mn1);
                    l0 = (h2 == 0 ? l0 * al0 : l0) + p00 + p10;
                    l1 = (h2 == 0 ? l1 * al1 : l1) + p01 + p11;
                    const uint32_t u0 = pack_bf16x2(p00, p01), u1 = pack_bf16x2(p10, p11);
                    const float2 f0 = unpack_bf16x2(u0), f1 = unpack_bf16x2(u1);
                    ph[h2][0] = movmatrix_t(u0);
                    ph[h2][1] = movmatrix_t(u1);
                    pl[h2][0] = movmatrix_t(pack_bf16x2(p00 - f0.x, p01 - f0.y));
                    pl[h2][1] = movmatrix_t(pack_bf16x2(p10 - f1.x, p11 - f1.y));
                }
#pragma unroll
                for (int mt = 0; mt < HD / 16; mt++) {
                    acc[mt][0] *= al0;
                    acc[mt][1] *= al1;
                    acc[mt][2] *= al0;
                    acc[mt][3] *= al1;
                }
#pragma unroll
                for (int mt = 0; mt < HD / 16; mt++) {
#pragma unroll
                    for (int h2 = 0; h2 < 2; h2++) {
                        uint32_t a0, a1, a2, a3;
                        const int vrow = h2 * 16 + (mi >> 1) * 8 + (lane & 7);
                        ldsm_x4_t(vb + (mt >> 2) * C::BOX_BYTES + sw128(vrow, 2 * (mt & 3) + (mi & 1)), a0, a1, a2,
                                  a3);
                        mma_bf16_16816(acc[mt], a0, a1, a2, a3, ph[h2][0], ph[h2][1]);
                        mma_bf16_16816(acc[mt], a0, a1, a2, a3, pl[h2][0], pl[h2][1]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_empty + 8 * st);
            ++ntile;
        }

        const bool last = t == tb - 1;
        if (it.j == it.T - 1 || last) {
            // ---- segment end in this CTA: hand this warp's state to the merger and go on; the CTA's last segment
            //      end is merged by the consumer warps together, in stage memory (every tile is consumed by then) ----
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                l0 += __shfl_xor_sync(0xffffffffu, l0, o);
                l1 += __shfl_xor_sync(0xffffffffu, l1, o);
            }
            float *Fb;
            if (last) {
                bar_consumers();  // all consumer warps are past their last tile: the stages are free
                Fb = reinterpret_cast<float *>(sm);
            } else {
                const int b = nflush % NFB;
                if (nflush >= NFB) {
                    const bool ok = __all_sync(0xffffffffu, misc[0] == 0 &&
                                                                mbar_wait(bar_fempty + 8 * b, (nflush / NFB - 1) & 1));
                    if (!ok) misc[0] = 1;
                }
                Fb = flush + b * NCW * C::PART_FLOATS;
            }
            float *F = Fb + warp * C::PART_FLOATS;
            if (lane < 4) {
                F[c2] = m0;
                F[c2 + 1] = m1;
                F[GMAX + c2] = l0;
                F[GMAX + c2 + 1] = l1;
            }
            float *O = F + 2 * GMAX;
#pragma unroll
            for (int mt = 0; mt < HD / 16; mt++) {
                const int d = mt * 16 + r4;
                O[c2 * HD + d] = acc[mt][0];
                O[(c2 + 1) * HD + d] = acc[mt][1];
                O[c2 * HD + d + 8] = acc[mt][2];
                O[(c2 + 1) * HD + d + 8] = acc[mt][3];
            }
            if (last) {
                bar_consumers();
                const long Sg = pre[it.s] + static_cast<long>(it.kh) * it.T;
                merge_segment<HD, NCW * 32>(P, Fb, it.s, it.kh, Sg, Sg + it.T, ta, tb, W, Gc, c,
                                            nflush == 0 ? 0 : 1, threadIdx.x, misc + 1, [] {});
            } else {
                __syncwarp();
                if (lane == 0) mbar_arrive(bar_ffull + 8 * (nflush % NFB));
            }
            nflush++;
            m0 = m1 = -INFINITY;
            l0 = l1 = 0.f;
#pragma unroll
            for (int mt = 0; mt < HD / 16; mt++) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
            need_q = true;
        }
        if (t + 1 < tb) it.next(Ls, nk);
        if (++owner == NCW) owner = 0;
    }
    if constexpr (DROP) {
        __syncwarp();
        bar_end_arrive();
    }
}

}  // namespace dec
