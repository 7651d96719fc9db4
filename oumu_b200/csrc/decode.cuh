// Split-KV GQA decode attention for sm_100a with the cross-split combine fused in.
//
// Work unit: a tile of 64 KV positions of one (take, kv head) "segment". All tiles of all segments are laid end to
// end (take-major, then kv head, then position) and cut into gridDim.x equal contiguous ranges, one per CTA, so
// every CTA streams the same number of bytes whatever the per-take lengths are. A CTA keeps one running
// online-softmax state per segment it touches; a segment entirely inside one CTA is finished there, a segment
// split across CTAs leaves one partial per CTA and the last CTA to finish (atomic counter, no waiting) merges them.
//
// Per CTA: one producer warp streams K and V tiles with TMA (128-byte swizzle) into a ring of shared-memory
// stages; four consumer warps each take 16 positions of a tile and run
//   S^T[16 pos x 8 heads] = K[16 x hd] . Q^T[hd x 8]        (mma.sync m16n8k16, A = K via ldmatrix, B = q in regs)
//   online softmax down the position axis (fp32, exp2 with the scale folded)
//   O^T[hd x 8 heads] += V^T[hd x 16] . P^T[16 x 8]          (A = V via ldmatrix.trans, B = P via movmatrix)
// so each KV byte is read from HBM once for all q heads of its GQA group (the reference reads it once per q head,
// kernels/voxcpm.cu:139-148).
#pragma once
#include "common.cuh"

namespace dec {

constexpr int TILE = 64;     // KV positions per stage
constexpr int NCW = 4;       // consumer warps (16 positions each)
constexpr int NTHREADS = (NCW + 1) * 32;
constexpr int GMAX = 8;      // q heads per kv head handled by one mma column block

template <int HD>
struct Cfg {
    static constexpr int NBOX = HD / 64;                   // 64-element (128-byte) TMA boxes per row
    static constexpr int BOX_BYTES = TILE * 128;           // 64 rows x 128 B
    static constexpr int KV_BYTES = NBOX * BOX_BYTES;      // one K (or V) tile
    static constexpr int STAGE_BYTES = 2 * KV_BYTES;
    static constexpr int PART_FLOATS = 2 * GMAX + GMAX * HD;  // m[8], l[8], o[8][HD]
    static constexpr int FLUSH_BYTES = NCW * PART_FLOATS * 4;
};

struct Params {
    const bf16 *qkv;
    bf16 *out;
    float *part;   // [gridDim.x][2][PART_FLOATS]
    int *cnt;      // [B * nk], zero between launches
    const int *pos;
    const int *lens;
    int B, nq, nk, maxlen, stages;
    float sl2;     // scale * log2(e)
};

// Shared-memory layout helper (offsets from the 1024-aligned base).
template <int HD>
struct Smem {
    int stages, B;
    __host__ __device__ int flush_off() const { return stages * Cfg<HD>::STAGE_BYTES; }
    __host__ __device__ int bar_off() const { return flush_off() + Cfg<HD>::FLUSH_BYTES; }
    __host__ __device__ int pre_off() const { return bar_off() + 2 * stages * 8; }
    __host__ __device__ int len_off() const { return pre_off() + (B + 1) * 4; }
    __host__ __device__ int misc_off() const { return len_off() + B * 4; }
    __host__ __device__ int bytes() const { return misc_off() + 16; }
};

// Position iterator over the tiles of the segments: segment (s, kh), tile j.
struct TileIt {
    int s, kh, j, T, L;
    __device__ void seek(long t, const int *pre, const int *Ls, int B, int nk) {
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

// CTA whose tile range contains tile t (ranges [c*W/G, (c+1)*W/G)).
__device__ __forceinline__ int cta_of(long t, long W, int G) {
    return static_cast<int>(((t + 1) * G + W - 1) / W) - 1;
}

template <int HD>
__global__ void __launch_bounds__(NTHREADS, 1)
    k_attn_decode(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv, Params P) {
    using C = Cfg<HD>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_s = smem_u32(smem_raw);
    uint8_t *sm = smem_raw + ((1024u - (raw_s & 1023u)) & 1023u);
    const uint32_t sm_s = smem_u32(sm);
    const Smem<HD> L{P.stages, P.B};
    float *flush = reinterpret_cast<float *>(sm + L.flush_off());
    const uint32_t bar_full = sm_s + L.bar_off();
    const uint32_t bar_empty = bar_full + 8 * P.stages;
    int *pre = reinterpret_cast<int *>(sm + L.pre_off());
    int *Ls = reinterpret_cast<int *>(sm + L.len_off());
    volatile int *misc = reinterpret_cast<volatile int *>(sm + L.misc_off());

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int B = P.B, nk = P.nk, G = P.nq / P.nk;

    // ---- per-take lengths and the tile prefix over takes (warp 0) ----
    if (warp == 0) {
        const int per = (B + 31) / 32, s0 = lane * per;
        int sum = 0;
        for (int k = 0; k < per; k++) {
            int s = s0 + k;
            if (s < B) {
                int Lv = P.lens ? P.lens[s] : *P.pos + 1;
                if (Lv < 1 || Lv > P.maxlen) {
                    record_error(OUMU_DEVERR_LENGTH);
                    Lv = Lv < 1 ? 1 : P.maxlen;
                }
                Ls[s] = Lv;
                sum += ((Lv + TILE - 1) / TILE) * nk;
            }
        }
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
        for (int i = 0; i < P.stages; i++) {
            mbar_init(bar_full + 8 * i, 1);
            mbar_init(bar_empty + 8 * i, NCW);
        }
        misc[0] = 0;  // abort flag
        mbar_fence_init();
    }
    __syncthreads();

    const long W = pre[B];
    const int Gc = gridDim.x, c = blockIdx.x;
    const long ta = static_cast<long>(c) * W / Gc, tb = static_cast<long>(c + 1) * W / Gc;
    if (ta >= tb) return;

    if (warp == NCW) {
        // ------------------------------ producer ------------------------------
        if (lane == 0) {
            tma_prefetch_desc(&tk);
            tma_prefetch_desc(&tv);
            TileIt it;
            it.seek(ta, pre, Ls, B, nk);
            for (long t = ta, i = 0; t < tb; t++, i++) {
                const int st = static_cast<int>(i % P.stages);
                const uint32_t use = static_cast<uint32_t>(i / P.stages);
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
            }
        }
        return;
    }

    // ------------------------------ consumers ------------------------------
    const int tid = threadIdx.x;  // 0 .. NCW*32-1
    const int r4 = lane >> 2, c2 = (lane & 3) * 2;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float acc[HD / 16][4];
#pragma unroll
    for (int mt = 0; mt < HD / 16; mt++) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
    uint32_t qb[HD / 16][2];
    bool need_q = true;
    int nflush = 0;

    TileIt it;
    it.seek(ta, pre, Ls, B, nk);
    for (long t = ta, i = 0; t < tb; t++, i++) {
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
            need_q = false;
        }
        const int st = static_cast<int>(i % P.stages);
        const uint32_t use = static_cast<uint32_t>(i / P.stages);
        bool ok = misc[0] == 0;
        if (ok && !mbar_wait(bar_full + 8 * st, use & 1u)) {
            misc[0] = 1;
            ok = false;
        }
        ok = __all_sync(0xffffffffu, ok);
        const int p0 = it.j * TILE + warp * 16;
        if (ok && p0 < it.L) {
            const uint32_t kb = sm_s + st * C::STAGE_BYTES, vb = kb + C::KV_BYTES;
            // S^T = K . Q^T, two accumulators to halve the dependency chain
            float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
            const int mi = lane >> 3;
            const int krow = warp * 16 + (mi & 1) * 8 + (lane & 7);
#pragma unroll
            for (int ks = 0; ks < HD / 16; ks++) {
                uint32_t a0, a1, a2, a3;
                ldsm_x4(kb + (ks >> 2) * C::BOX_BYTES + sw128(krow, 2 * (ks & 3) + (mi >> 1)), a0, a1, a2, a3);
                mma_bf16_16816((ks & 1) ? sb : sa, a0, a1, a2, a3, qb[ks][0], qb[ks][1]);
            }
            float x[4];
#pragma unroll
            for (int k = 0; k < 4; k++) x[k] = (sa[k] + sb[k]) * P.sl2;
            const int pr0 = p0 + r4, pr1 = pr0 + 8;
            if (pr0 >= it.L) x[0] = x[1] = -INFINITY;
            if (pr1 >= it.L) x[2] = x[3] = -INFINITY;
            float mx0 = fmaxf(x[0], x[2]), mx1 = fmaxf(x[1], x[3]);
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
            }
            const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
            const float al0 = fast_exp2(m0 - mn0), al1 = fast_exp2(m1 - mn1);
            m0 = mn0;
            m1 = mn1;
            const float p00 = fast_exp2(x[0] - mn0), p01 = fast_exp2(x[1] - mn1);
            const float p10 = fast_exp2(x[2] - mn0), p11 = fast_exp2(x[3] - mn1);
            l0 = l0 * al0 + p00 + p10;
            l1 = l1 * al1 + p01 + p11;
#pragma unroll
            for (int mt = 0; mt < HD / 16; mt++) {
                acc[mt][0] *= al0;
                acc[mt][1] *= al1;
                acc[mt][2] *= al0;
                acc[mt][3] *= al1;
            }
            const uint32_t pb0 = movmatrix_t(pack_bf16x2(p00, p01));
            const uint32_t pb1 = movmatrix_t(pack_bf16x2(p10, p11));
            const int vrow = warp * 16 + (mi >> 1) * 8 + (lane & 7);
#pragma unroll
            for (int mt = 0; mt < HD / 16; mt++) {
                uint32_t a0, a1, a2, a3;
                ldsm_x4_t(vb + (mt >> 2) * C::BOX_BYTES + sw128(vrow, 2 * (mt & 3) + (mi & 1)), a0, a1, a2, a3);
                mma_bf16_16816(acc[mt], a0, a1, a2, a3, pb0, pb1);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_empty + 8 * st);

        if (it.j == it.T - 1 || t == tb - 1) {
            // ---------------- segment (s, kh) ends in this CTA: merge the warps ----------------
            const int s = it.s, kh = it.kh, g = s * nk + kh;
            const long Sg = pre[s] + static_cast<long>(kh) * it.T, Eg = Sg + it.T;
            const bool whole = Sg >= ta && Eg <= tb;
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                l0 += __shfl_xor_sync(0xffffffffu, l0, o);
                l1 += __shfl_xor_sync(0xffffffffu, l1, o);
            }
            float *F = flush + warp * C::PART_FLOATS;
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
            bar_consumers();
            constexpr int TPH = HD / 8;  // threads per head, 8 outputs each
            const int h = tid / TPH, d0 = (tid % TPH) * 8;
            float Mx = -INFINITY, Lsum = 0.f, o[8];
#pragma unroll
            for (int k = 0; k < 8; k++) o[k] = 0.f;
            if (h < GMAX) {
#pragma unroll
                for (int w = 0; w < NCW; w++) Mx = fmaxf(Mx, flush[w * C::PART_FLOATS + h]);
#pragma unroll
                for (int w = 0; w < NCW; w++) {
                    const float *Fw = flush + w * C::PART_FLOATS;
                    const float mw = Fw[h];
                    const float cw = mw == -INFINITY ? 0.f : fast_exp2(mw - Mx);
                    Lsum += cw * Fw[GMAX + h];
                    const float *ow = Fw + 2 * GMAX + h * HD + d0;
#pragma unroll
                    for (int k = 0; k < 8; k++) o[k] += cw * ow[k];
                }
            }
            bf16 *dst = P.out + static_cast<long>(s) * P.nq * HD + (kh * G + h) * HD + d0;
            if (whole) {
                if (h < G) {
                    uint4 u;
                    uint32_t *uw = reinterpret_cast<uint32_t *>(&u);
#pragma unroll
                    for (int k = 0; k < 4; k++) uw[k] = pack_bf16x2(o[2 * k] / Lsum, o[2 * k + 1] / Lsum);
                    *reinterpret_cast<uint4 *>(dst) = u;
                }
            } else {
                const int slot = nflush == 0 ? 0 : 1;
                float *rec = P.part + (static_cast<long>(c) * 2 + slot) * C::PART_FLOATS;
                if (h < GMAX) {
                    if (d0 == 0) {
                        rec[h] = Mx;
                        rec[GMAX + h] = Lsum;
                    }
                    float4 *ro = reinterpret_cast<float4 *>(rec + 2 * GMAX + h * HD + d0);
                    ro[0] = make_float4(o[0], o[1], o[2], o[3]);
                    ro[1] = make_float4(o[4], o[5], o[6], o[7]);
                }
                __threadfence();
                bar_consumers();
                if (tid == 0) misc[1] = atomicAdd(P.cnt + g, 1);
                bar_consumers();
                const int cf = cta_of(Sg, W, Gc), cl = cta_of(Eg - 1, W, Gc);
                if (misc[1] == cl - cf) {
                    // last contributor: merge every CTA's partial of this segment
                    __threadfence();
                    if (h < G) {
                        float M2 = -INFINITY;
                        for (int cc = cf; cc <= cl; cc++) {
                            const long ac = static_cast<long>(cc) * W / Gc;
                            const int sl = (cc == cf && ac < Sg) ? 1 : 0;
                            M2 = fmaxf(M2, __ldcg(P.part + (static_cast<long>(cc) * 2 + sl) * C::PART_FLOATS + h));
                        }
                        float L2 = 0.f, o2[8];
#pragma unroll
                        for (int k = 0; k < 8; k++) o2[k] = 0.f;
                        for (int cc = cf; cc <= cl; cc++) {
                            const long ac = static_cast<long>(cc) * W / Gc;
                            const int sl = (cc == cf && ac < Sg) ? 1 : 0;
                            const float *rc = P.part + (static_cast<long>(cc) * 2 + sl) * C::PART_FLOATS;
                            const float mc = __ldcg(rc + h);
                            const float wc = mc == -INFINITY ? 0.f : fast_exp2(mc - M2);
                            L2 += wc * __ldcg(rc + GMAX + h);
                            const float4 *oc = reinterpret_cast<const float4 *>(rc + 2 * GMAX + h * HD + d0);
                            const float4 u0 = __ldcg(oc), u1 = __ldcg(oc + 1);
                            o2[0] += wc * u0.x; o2[1] += wc * u0.y; o2[2] += wc * u0.z; o2[3] += wc * u0.w;
                            o2[4] += wc * u1.x; o2[5] += wc * u1.y; o2[6] += wc * u1.z; o2[7] += wc * u1.w;
                        }
                        uint4 u;
                        uint32_t *uw = reinterpret_cast<uint32_t *>(&u);
#pragma unroll
                        for (int k = 0; k < 4; k++) uw[k] = pack_bf16x2(o2[2 * k] / L2, o2[2 * k + 1] / L2);
                        *reinterpret_cast<uint4 *>(dst) = u;
                    }
                    if (tid == 0) P.cnt[g] = 0;
                }
                nflush++;
            }
            if (whole) nflush++;
            bar_consumers();
            m0 = m1 = -INFINITY;
            l0 = l1 = 0.f;
#pragma unroll
            for (int mt = 0; mt < HD / 16; mt++) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
            need_q = true;
        }
        if (t + 1 < tb) it.next(Ls, nk);
    }
}

}  // namespace dec
