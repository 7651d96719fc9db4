// Attention feeders: rotary embedding, KV-cache writes and slot replication.
// All of them move 16-byte vectors; the arithmetic of rope is the reference's, term for term, so results are
// bit-identical to kernels/voxcpm.cu:100-129,407-413.
#pragma once
#include "common.cuh"

// Rotate 8 consecutive pairs (x1 = v[i..i+8), x2 = v[i+half..i+half+8)) of one head in place, at table row p.
// Mirrors kernels/voxcpm.cu:109-114: x1' = bf16(x1*c - x2*s), x2' = bf16(x2*c + x1*s).
__device__ __forceinline__ void rope8(bf16 *v, int i, int half, const float *cos_t, const float *sin_t, long p,
                                      uint4 *k_out) {
    uint4 u1 = *reinterpret_cast<const uint4 *>(v + i);
    uint4 u2 = *reinterpret_cast<const uint4 *>(v + i + half);
    const float4 *cp = reinterpret_cast<const float4 *>(cos_t + p * half + i);
    const float4 *sp = reinterpret_cast<const float4 *>(sin_t + p * half + i);
    float4 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
    float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    float s[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const bf16 *a = reinterpret_cast<const bf16 *>(&u1);
    const bf16 *b = reinterpret_cast<const bf16 *>(&u2);
    uint4 o1, o2;
    bf16 *oa = reinterpret_cast<bf16 *>(&o1);
    bf16 *ob = reinterpret_cast<bf16 *>(&o2);
#pragma unroll
    for (int j = 0; j < 8; j++) {
        float x1 = bf2f(a[j]), x2 = bf2f(b[j]);
        oa[j] = f2bf(x1 * c[j] - x2 * s[j]);
        ob[j] = f2bf(x2 * c[j] + x1 * s[j]);
    }
    *reinterpret_cast<uint4 *>(v + i) = o1;
    *reinterpret_cast<uint4 *>(v + i + half) = o2;
    if (k_out) {
        k_out[0] = o1;
        k_out[1] = o2;
    }
}

// One thread per (row, head, group of 8 pairs). Position: r % seq (seq > 0) or *pos (kernels/voxcpm.cu:106).
__global__ void __launch_bounds__(256) k_rope(bf16 *qkv, const float *cos_t, const float *sin_t, const int *pos,
                                              int rows, int seq, int nq, int nk, int hd) {
    const int half = hd / 2, groups = half / 8, heads = nq + nk;
    long t = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= static_cast<long>(rows) * heads * groups) return;
    int g = static_cast<int>(t % groups);
    long rh = t / groups;
    int h = static_cast<int>(rh % heads);
    int r = static_cast<int>(rh / heads);
    int p = seq > 0 ? r % seq : *pos;
    bf16 *v = qkv + static_cast<long>(r) * (nq + 2 * nk) * hd + h * hd;
    rope8(v, g * 8, half, cos_t, sin_t, p, nullptr);
}

// One thread per 16-byte chunk of k or v: grid covers slots * rows * nk * (hd/8) * 2 chunks.
// Addressing of kernels/voxcpm.cu:121-127: dst = ((s*nk + h)*maxlen + p)*hd, src row s*rows + i.
__global__ void __launch_bounds__(256) k_kv_write(const bf16 *qkv, bf16 *kc, bf16 *vc, const int *pos, int slots,
                                                  int rows, int nq, int nk, int hd, int maxlen) {
    const int cpr = hd / 8;  // 16-byte chunks per head row
    long t = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
    long total = static_cast<long>(slots) * rows * nk * cpr * 2;
    if (t >= total) return;
    int c = static_cast<int>(t % cpr);
    long r = t / cpr;
    int h = static_cast<int>(r % nk);
    r /= nk;
    int which = static_cast<int>(r % 2);  // 0 = k, 1 = v
    r /= 2;
    int i = static_cast<int>(r % rows);
    int s = static_cast<int>(r / rows);
    int p = (pos ? *pos : 0) + i;
    const bf16 *src = qkv + (static_cast<long>(s) * rows + i) * (nq + 2 * nk) * hd + (nq + which * nk + h) * hd;
    bf16 *dst = (which ? vc : kc) + ((static_cast<long>(s) * nk + h) * maxlen + p) * hd;
    reinterpret_cast<uint4 *>(dst)[c] = reinterpret_cast<const uint4 *>(src)[c];
}

// Decode prologue: one block per take. Threads [0, (nq+nk)*half/8) rotate q and k (k also written to the cache),
// the next nk*hd/8 threads copy v. Position p_s = lens[s]-1 or *pos.
__global__ void __launch_bounds__(256) k_decode_prologue(bf16 *qkv, bf16 *kc, bf16 *vc, const float *cos_t,
                                                         const float *sin_t, const int *pos, const int *lens, int nq,
                                                         int nk, int hd, int maxlen) {
    const int s = blockIdx.x, half = hd / 2, groups = half / 8;
    if (threadIdx.x == 0) pdl_trigger();
    pdl_wait();
    int p = lens ? lens[s] - 1 : *pos;
    if (p < 0 || p >= maxlen) {
        if (threadIdx.x == 0) record_error(OUMU_DEVERR_LENGTH);
        return;
    }
    bf16 *row = qkv + static_cast<long>(s) * (nq + 2 * nk) * hd;
    const int nrot = (nq + nk) * groups, ncopy = nk * (hd / 8);
    for (int t = threadIdx.x; t < nrot + ncopy; t += blockDim.x) {
        if (t < nrot) {
            int h = t / groups, g = t % groups;
            bf16 *v = row + h * hd;
            if (h >= nq) {
                bf16 *dst = kc + ((static_cast<long>(s) * nk + (h - nq)) * maxlen + p) * hd;
                if (cos_t) {
                    uint4 o[2];
                    rope8(v, g * 8, half, cos_t, sin_t, p, o);
                    reinterpret_cast<uint4 *>(dst + g * 8)[0] = o[0];
                    reinterpret_cast<uint4 *>(dst + g * 8 + half)[0] = o[1];
                } else {
                    reinterpret_cast<uint4 *>(dst + g * 8)[0] = reinterpret_cast<const uint4 *>(v + g * 8)[0];
                    reinterpret_cast<uint4 *>(dst + g * 8 + half)[0] =
                        reinterpret_cast<const uint4 *>(v + g * 8 + half)[0];
                }
            } else if (cos_t) {
                rope8(v, g * 8, half, cos_t, sin_t, p, nullptr);
            }
        } else {
            int u = t - nrot, h = u / (hd / 8), c = u % (hd / 8);
            const bf16 *src = row + (nq + nk + h) * hd;
            bf16 *dst = vc + ((static_cast<long>(s) * nk + h) * maxlen + p) * hd;
            reinterpret_cast<uint4 *>(dst)[c] = reinterpret_cast<const uint4 *>(src)[c];
        }
    }
}

// Slot 0 -> slots 1..B-1 for positions < T (kernels/voxcpm.cu:407-413). One thread per 16-byte chunk of a
// (position, head) row of slot 0; blockIdx.y selects a group of destination slots.
__global__ void __launch_bounds__(256) k_kv_replicate(bf16 *c, int B, int nk, int maxlen, int hd, int T,
                                                      int slots_per_group) {
    const int cpr = hd / 8;
    long t = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= static_cast<long>(T) * nk * cpr) return;
    int ch = static_cast<int>(t % cpr);
    long ph = t / cpr;
    int h = static_cast<int>(ph % nk);
    int p = static_cast<int>(ph / nk);
    uint4 v = reinterpret_cast<const uint4 *>(c + (static_cast<long>(h) * maxlen + p) * hd)[ch];
    int s0 = 1 + blockIdx.y * slots_per_group;
    int s1 = min(B, s0 + slots_per_group);
    for (int s = s0; s < s1; s++)
        reinterpret_cast<uint4 *>(c + ((static_cast<long>(s) * nk + h) * maxlen + p) * hd)[ch] = v;
}
