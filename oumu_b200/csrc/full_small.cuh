// Attention inside many short independent sequences (seq <= 16): the LocDiT passes (11 or 12 tokens, all takes x
// both CFG branches in one launch) and the local encoder (5 tokens).
//
// k_attn_small (one q head per kv head): one warp per (sequence, q head) unit, persistent over units. The warp stages
// its q, k and v rows (16-byte cp.async, 128-byte-swizzled rows, padding rows zeroed) in its own shared-memory slice,
// then on tensor cores:
//   S[16 x 16] = Q[16 x hd] . K^T          (mma.sync m16n8k16, fp32 accumulate)
//   row softmax in fp32 (exp2 with the scale folded), masked keys (>= seq, or causal) -> 0
//   O[16 x hd] = P . V                       (P split as bf16 hi + lo, so the weights keep ~16 mantissa bits)
//   out = bf16(O * (1 / sum))                the reference's normalisation point (kernels/voxcpm.cu:291-295)
#pragma once
#include "common.cuh"

namespace fs {

constexpr int WARPS = 4;
constexpr int ROWS = 16;

template <int HD>
struct Cfg {
    static constexpr int NBOX = HD / 64;
    static constexpr int MAT_BYTES = NBOX * ROWS * 128;   // one 16-row matrix, 128-B swizzled rows per box
    static constexpr int WARP_BYTES = 3 * MAT_BYTES;      // q, k, v
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <int HD>
__global__ void __launch_bounds__(WARPS * 32) k_attn_small(const bf16 *__restrict__ qkv, bf16 *__restrict__ out,
                                                           int nseq, int seq, int causal, int nq, int nk,
                                                           float sl2) {
    using C = Cfg<HD>;
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t *ws = smem + warp * C::WARP_BYTES;
    const uint32_t ws_s = smem_u32(ws);
    const int stride = (nq + 2 * nk) * HD, G = nq / nk;
    const int CPR = HD / 8;  // 16-byte chunks per row
    const long units = static_cast<long>(nseq) * nq;
    const int r4 = lane >> 2, c2 = (lane & 3) * 2, mi = lane >> 3;

    for (long u = static_cast<long>(blockIdx.x) * WARPS + warp; u < units; u += static_cast<long>(gridDim.x) * WARPS) {
        const int n = static_cast<int>(u / nq), h = static_cast<int>(u % nq), kh = h / G;
        const bf16 *base = qkv + static_cast<long>(n) * seq * stride;
        // ---- stage q, k, v rows (rows >= seq zero-filled) ----
        for (int i = lane; i < 3 * ROWS * CPR; i += 32) {
            const int mat = i / (ROWS * CPR), rem = i % (ROWS * CPR), r = rem / CPR, ch = rem % CPR;
            const uint32_t dst = ws_s + mat * C::MAT_BYTES + (ch >> 3) * (ROWS * 128) + sw128(r, ch & 7);
            if (r < seq) {
                const int col = mat == 0 ? h * HD : (mat == 1 ? (nq + kh) * HD : (nq + nk + kh) * HD);
                cp_async16(dst, base + static_cast<long>(r) * stride + col + ch * 8);
            } else {
                asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dst), "r"(0) : "memory");
            }
        }
        cp_async_wait_all();
        __syncwarp();
        const uint32_t qs = ws_s, ks_ = ws_s + C::MAT_BYTES, vs = ws_s + 2 * C::MAT_BYTES;

        // ---- S = Q K^T ----
        float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int ks = 0; ks < HD / 16; ks++) {
            uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
            const uint32_t boff = (ks >> 2) * (ROWS * 128);
            ldsm_x4(qs + boff + sw128((mi & 1) * 8 + (lane & 7), 2 * (ks & 3) + (mi >> 1)), a0, a1, a2, a3);
            ldsm_x4(ks_ + boff + sw128((mi >> 1) * 8 + (lane & 7), 2 * (ks & 3) + (mi & 1)), b0, b1, b2, b3);
            mma_bf16_16816(s[0], a0, a1, a2, a3, b0, b1);
            mma_bf16_16816(s[1], a0, a1, a2, a3, b2, b3);
        }
        // ---- masked row softmax (rows r4 and r4 + 8) ----
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int nt = 0; nt < 2; nt++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int row = r4 + (e >> 1) * 8, key = nt * 8 + c2 + (e & 1);
                const bool ok = key < seq && (!causal || key <= row);
                s[nt][e] = ok ? s[nt][e] * sl2 : -INFINITY;
                mx[e >> 1] = fmaxf(mx[e >> 1], s[nt][e]);
            }
#pragma unroll
        for (int k = 0; k < 2; k++) {
            mx[k] = fmaxf(mx[k], __shfl_xor_sync(0xffffffffu, mx[k], 1));
            mx[k] = fmaxf(mx[k], __shfl_xor_sync(0xffffffffu, mx[k], 2));
            if (mx[k] == -INFINITY) mx[k] = 0.f;  // padding rows only
        }
        float sum[2] = {0.f, 0.f};
#pragma unroll
        for (int nt = 0; nt < 2; nt++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                s[nt][e] = fast_exp2(s[nt][e] - mx[e >> 1]);
                sum[e >> 1] += s[nt][e];
            }
#pragma unroll
        for (int k = 0; k < 2; k++) {
            sum[k] += __shfl_xor_sync(0xffffffffu, sum[k], 1);
            sum[k] += __shfl_xor_sync(0xffffffffu, sum[k], 2);
        }
        // P as the A operand (k = keys): a0 = row r4 keys 0-7, a1 = row r4+8 keys 0-7, a2/a3 keys 8-15; hi + lo parts
        uint32_t ph[4], pl[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int nt = k >> 1, e = (k & 1) * 2;
            const float x0 = s[nt][e], x1 = s[nt][e + 1];
            ph[k] = pack_bf16x2(x0, x1);
            const float2 hv = unpack_bf16x2(ph[k]);
            pl[k] = pack_bf16x2(x0 - hv.x, x1 - hv.y);
        }
        // ---- O = P V, two d-tiles of 8 per ldmatrix.x4.trans ----
        const float inv0 = 1.f / sum[0], inv1 = 1.f / sum[1];
        const int row0 = r4, row1 = r4 + 8;
        bf16 *o0 = out + (static_cast<long>(n) * seq + row0) * nq * HD + h * HD;
        bf16 *o1 = out + (static_cast<long>(n) * seq + row1) * nq * HD + h * HD;
#pragma unroll
        for (int dt = 0; dt < HD / 8; dt += 2) {
            uint32_t b0, b1, b2, b3;
            const int ch = dt + (mi >> 1);
            ldsm_x4_t(vs + (ch >> 3) * (ROWS * 128) + sw128((mi & 1) * 8 + (lane & 7), ch & 7), b0, b1, b2, b3);
            float o[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
            mma_bf16_16816(o[0], ph[0], ph[1], ph[2], ph[3], b0, b1);
            mma_bf16_16816(o[0], pl[0], pl[1], pl[2], pl[3], b0, b1);
            mma_bf16_16816(o[1], ph[0], ph[1], ph[2], ph[3], b2, b3);
            mma_bf16_16816(o[1], pl[0], pl[1], pl[2], pl[3], b2, b3);
#pragma unroll
            for (int t = 0; t < 2; t++) {
                const int d = (dt + t) * 8 + c2;
                if (row0 < seq)
                    *reinterpret_cast<uint32_t *>(o0 + d) = pack_bf16x2(o[t][0] * inv0, o[t][1] * inv0);
                if (row1 < seq)
                    *reinterpret_cast<uint32_t *>(o1 + d) = pack_bf16x2(o[t][2] * inv1, o[t][3] * inv1);
            }
        }
        __syncwarp();
    }
}

// ------------------------------------------------------------------------------------------------------------
// k_attn_small_grp (grouped-query attention, G = nq / nk > 1, G * seq <= 128): one CTA per (sequence, kv head).
// The G q heads of the group are stacked as one tall Q (row g * seq + r = head g, query r; padded to MT 16-row
// tiles); the CTA stages K and V once and the whole stack (every byte read from memory once per group, not once
// per q head), then warp t computes Q tile t: S = Q_t K^T, masked row softmax, O = P V, out = bf16(O * (1 / sum)) —
// the arithmetic of k_attn_small row for row.
// ROPE: q and k are rotated while they are staged (position r of the sequence, the arithmetic of k_rope:
// x1' = bf16(x1*c - x2*s), x2' = bf16(x2*c + x1*s)), so one launch replaces rope + attention of Engine::full
// (src/model.rs:541-567) with the same result; qkv itself is left unrotated.
// ------------------------------------------------------------------------------------------------------------
constexpr int MAXM = 128;  // stacked q rows at most: MT <= 8 warps

template <int HD>
struct GCfg {
    static constexpr int NBOX = HD / 64;
    static constexpr int TILE_BYTES = NBOX * ROWS * 128;  // one 16-row matrix, 128-B swizzled rows per 64-wide box
    static constexpr int smem_bytes(int mt) { return (2 + mt) * TILE_BYTES; }  // K, V, the Q tiles
};

// Stage one rotated chunk pair of a q or k row: chunks p and p + HD/16 (elements [8p, 8p+8) and the same + HD/2)
// rotated with the table row `pos`, stored into a 16-row swizzled matrix at row r.
template <int HD>
__device__ __forceinline__ void stage_rope_pair(uint32_t mat, int r, int p, const bf16 *row, const float *cos_t,
                                                const float *sin_t, int pos) {
    constexpr int HALF = HD / 2, HP = HD / 16;
    const uint4 u1 = *reinterpret_cast<const uint4 *>(row + p * 8);
    const uint4 u2 = *reinterpret_cast<const uint4 *>(row + HALF + p * 8);
    const float4 *cp = reinterpret_cast<const float4 *>(cos_t + static_cast<long>(pos) * HALF + p * 8);
    const float4 *sp = reinterpret_cast<const float4 *>(sin_t + static_cast<long>(pos) * HALF + p * 8);
    const float4 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
    const float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const bf16 *a = reinterpret_cast<const bf16 *>(&u1);
    const bf16 *b = reinterpret_cast<const bf16 *>(&u2);
    uint4 o1, o2;
    bf16 *oa = reinterpret_cast<bf16 *>(&o1);
    bf16 *ob = reinterpret_cast<bf16 *>(&o2);
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float x1 = bf2f(a[j]), x2 = bf2f(b[j]);
        oa[j] = f2bf(x1 * c[j] - x2 * sn[j]);
        ob[j] = f2bf(x2 * c[j] + x1 * sn[j]);
    }
    const int q = p + HP;  // the partner chunk
    st_shared_v4(mat + (p >> 3) * (ROWS * 128) + sw128(r, p & 7), o1);
    st_shared_v4(mat + (q >> 3) * (ROWS * 128) + sw128(r, q & 7), o2);
}

template <int HD, bool ROPE>
__global__ void __launch_bounds__(MAXM / ROWS * 32) k_attn_small_grp(const bf16 *__restrict__ qkv,
                                                                     bf16 *__restrict__ out, int seq, int causal,
                                                                     int nq, int nk, float sl2,
                                                                     const float *__restrict__ cos_t,
                                                                     const float *__restrict__ sin_t) {
    using C = GCfg<HD>;
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nthr = blockDim.x;
    const uint32_t ks_ = smem_u32(smem), vs = ks_ + C::TILE_BYTES, qs0 = vs + C::TILE_BYTES;
    const int stride = (nq + 2 * nk) * HD, G = nq / nk;
    const int CPR = HD / 8;  // 16-byte chunks per row
    const int M = G * seq, MT = nthr / 32;
    const int n = blockIdx.x / nk, kh = blockIdx.x % nk;
    const bf16 *base = qkv + static_cast<long>(n) * seq * stride;
    const int r4 = lane >> 2, c2 = (lane & 3) * 2, mi = lane >> 3;

    // ---- stage k, v (16 rows, zero past seq) and the stacked q rows (MT * 16, zero past M) ----
    if constexpr (ROPE) {
        // v by 16-byte chunks (cp.async); k and q by rotated chunk pairs through registers
        constexpr int HP = HD / 16;
        const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
        const int vitems = ROWS * CPR, kitems = ROWS * HP;
        for (int i = threadIdx.x; i < vitems + kitems + MT * ROWS * HP; i += nthr) {
            if (i < vitems) {
                const int r = i / CPR, ch = i % CPR;
                const uint32_t dst = vs + (ch >> 3) * (ROWS * 128) + sw128(r, ch & 7);
                if (r < seq) cp_async16(dst, base + static_cast<long>(r) * stride + (nq + nk + kh) * HD + ch * 8);
                else st_shared_v4(dst, zero);
            } else if (i < vitems + kitems) {
                const int j = i - vitems, r = j / HP, p = j % HP;
                if (r < seq) {
                    stage_rope_pair<HD>(ks_, r, p, base + static_cast<long>(r) * stride + (nq + kh) * HD, cos_t,
                                        sin_t, r);
                } else {
                    st_shared_v4(ks_ + (p >> 3) * (ROWS * 128) + sw128(r, p & 7), zero);
                    st_shared_v4(ks_ + ((p + HP) >> 3) * (ROWS * 128) + sw128(r, (p + HP) & 7), zero);
                }
            } else {
                const int j = i - vitems - kitems, m = j / HP, p = j % HP;
                const uint32_t mat = qs0 + (m >> 4) * C::TILE_BYTES;
                if (m < M) {
                    const int g = m / seq, r = m - g * seq;
                    stage_rope_pair<HD>(mat, m & 15, p, base + static_cast<long>(r) * stride + (kh * G + g) * HD,
                                        cos_t, sin_t, r);
                } else {
                    st_shared_v4(mat + (p >> 3) * (ROWS * 128) + sw128(m & 15, p & 7), zero);
                    st_shared_v4(mat + ((p + HP) >> 3) * (ROWS * 128) + sw128(m & 15, (p + HP) & 7), zero);
                }
            }
        }
    } else {
        const int kvitems = 2 * ROWS * CPR;
        for (int i = threadIdx.x; i < kvitems + MT * ROWS * CPR; i += nthr) {
            if (i < kvitems) {
                const int mat = i / (ROWS * CPR), rem = i % (ROWS * CPR), r = rem / CPR, ch = rem % CPR;
                const uint32_t dst = (mat == 0 ? ks_ : vs) + (ch >> 3) * (ROWS * 128) + sw128(r, ch & 7);
                if (r < seq) {
                    cp_async16(dst, base + static_cast<long>(r) * stride + (mat == 0 ? nq + kh : nq + nk + kh) * HD +
                                        ch * 8);
                } else {
                    asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dst), "r"(0) : "memory");
                }
            } else {
                const int j = i - kvitems, m = j / CPR, ch = j % CPR;
                const uint32_t dst =
                    qs0 + (m >> 4) * C::TILE_BYTES + (ch >> 3) * (ROWS * 128) + sw128(m & 15, ch & 7);
                if (m < M) {
                    const int g = m / seq, r = m - g * seq;
                    cp_async16(dst, base + static_cast<long>(r) * stride + (kh * G + g) * HD + ch * 8);
                } else {
                    asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dst), "r"(0) : "memory");
                }
            }
        }
    }
    cp_async_wait_all();
    __syncthreads();

    const uint32_t qs = qs0 + warp * C::TILE_BYTES;
    // ---- S = Q_t K^T ----
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int ks = 0; ks < HD / 16; ks++) {
        uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
        const uint32_t boff = (ks >> 2) * (ROWS * 128);
        ldsm_x4(qs + boff + sw128((mi & 1) * 8 + (lane & 7), 2 * (ks & 3) + (mi >> 1)), a0, a1, a2, a3);
        ldsm_x4(ks_ + boff + sw128((mi >> 1) * 8 + (lane & 7), 2 * (ks & 3) + (mi & 1)), b0, b1, b2, b3);
        mma_bf16_16816(s[0], a0, a1, a2, a3, b0, b1);
        mma_bf16_16816(s[1], a0, a1, a2, a3, b2, b3);
    }
    // ---- masked row softmax (stacked rows warp*16 + r4 and + 8) ----
    const int m0 = warp * 16 + r4, m1 = m0 + 8;
    const int q0 = m0 % seq, q1 = m1 % seq;  // query positions within the sequence
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 2; nt++)
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int qr = (e >> 1) ? q1 : q0, key = nt * 8 + c2 + (e & 1);
            const bool ok = key < seq && (!causal || key <= qr);
            s[nt][e] = ok ? s[nt][e] * sl2 : -INFINITY;
            mx[e >> 1] = fmaxf(mx[e >> 1], s[nt][e]);
        }
#pragma unroll
    for (int k = 0; k < 2; k++) {
        mx[k] = fmaxf(mx[k], __shfl_xor_sync(0xffffffffu, mx[k], 1));
        mx[k] = fmaxf(mx[k], __shfl_xor_sync(0xffffffffu, mx[k], 2));
        if (mx[k] == -INFINITY) mx[k] = 0.f;  // padding rows only
    }
    float sum[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < 2; nt++)
#pragma unroll
        for (int e = 0; e < 4; e++) {
            s[nt][e] = fast_exp2(s[nt][e] - mx[e >> 1]);
            sum[e >> 1] += s[nt][e];
        }
#pragma unroll
    for (int k = 0; k < 2; k++) {
        sum[k] += __shfl_xor_sync(0xffffffffu, sum[k], 1);
        sum[k] += __shfl_xor_sync(0xffffffffu, sum[k], 2);
    }
    uint32_t ph[4], pl[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int nt = k >> 1, e = (k & 1) * 2;
        const float x0 = s[nt][e], x1 = s[nt][e + 1];
        ph[k] = pack_bf16x2(x0, x1);
        const float2 hv = unpack_bf16x2(ph[k]);
        pl[k] = pack_bf16x2(x0 - hv.x, x1 - hv.y);
    }
    // ---- O = P V; stacked row m is query m % seq of q head kh * G + m / seq ----
    const float inv0 = 1.f / sum[0], inv1 = 1.f / sum[1];
    const bool st0 = m0 < M, st1 = m1 < M;
    bf16 *o0 = out + (static_cast<long>(n) * seq + q0) * nq * HD + (kh * G + m0 / seq) * HD;
    bf16 *o1 = out + (static_cast<long>(n) * seq + q1) * nq * HD + (kh * G + m1 / seq) * HD;
#pragma unroll
    for (int dt = 0; dt < HD / 8; dt += 2) {
        uint32_t b0, b1, b2, b3;
        const int ch = dt + (mi >> 1);
        ldsm_x4_t(vs + (ch >> 3) * (ROWS * 128) + sw128((mi & 1) * 8 + (lane & 7), ch & 7), b0, b1, b2, b3);
        float o[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        mma_bf16_16816(o[0], ph[0], ph[1], ph[2], ph[3], b0, b1);
        mma_bf16_16816(o[0], pl[0], pl[1], pl[2], pl[3], b0, b1);
        mma_bf16_16816(o[1], ph[0], ph[1], ph[2], ph[3], b2, b3);
        mma_bf16_16816(o[1], pl[0], pl[1], pl[2], pl[3], b2, b3);
#pragma unroll
        for (int tt = 0; tt < 2; tt++) {
            const int d = (dt + tt) * 8 + c2;
            if (st0) *reinterpret_cast<uint32_t *>(o0 + d) = pack_bf16x2(o[tt][0] * inv0, o[tt][1] * inv0);
            if (st1) *reinterpret_cast<uint32_t *>(o1 + d) = pack_bf16x2(o[tt][2] * inv1, o[tt][3] * inv1);
        }
    }
}

}  // namespace fs
