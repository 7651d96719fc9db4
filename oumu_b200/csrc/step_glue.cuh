// Element-wise and per-row kernels of the decoding step around the attention (the step's glue): RMS norms, the
// SwiGLU product, the DiT and local-encoder input sequences, classifier-free guidance with the Euler update, the
// FSQ activation and the step end. The norm, SwiGLU and pointwise kernels take part in programmatic dependent launch
// (oumu_set_pdl): they let the next kernel start at once and wait for the preceding one before touching its outputs. Each has the rounding points of the reference kernel it stands in for
// (kernels/voxcpm.cu), so a step built from them tracks the reference step; the layouts are this library's own:
// every kernel moves 16-byte vectors, and row norms run one block per row with the row held in registers.
#pragma once
#include "common.cuh"

namespace glue {

__device__ __forceinline__ float rbf(float x) { return bf2f(f2bf(x)); }

__device__ __forceinline__ void load8(const bf16 *p, float *v) {
    uint4 u = *reinterpret_cast<const uint4 *>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
        float2 f = unpack_bf16x2(w[j]);
        v[2 * j] = f.x;
        v[2 * j + 1] = f.y;
    }
}
__device__ __forceinline__ void store8(bf16 *p, const float *v) {
    uint4 u;
    u.x = pack_bf16x2(v[0], v[1]);
    u.y = pack_bf16x2(v[2], v[3]);
    u.z = pack_bf16x2(v[4], v[5]);
    u.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4 *>(p) = u;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// One block per row of DIM elements, DIM/8 threads, one 16-byte vector each: rows spread over the SMs, and the
// row, its residual and the norm weights are all in flight at once. With `d`: res = bf16(res + d) first
// (add_rmsnorm, kernels/voxcpm.cu:55-67), else rmsnorm (kernels/voxcpm.cu:43-52).
// out = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w).
template <int DIM>
__global__ void __launch_bounds__(DIM / 8) k_rmsnorm(bf16 *res, const bf16 *d, const bf16 *w, bf16 *out, int rows,
                                                     float eps) {
    constexpr int NW = DIM / 256;
    __shared__ float red[NW];
    const int c = threadIdx.x * 8;
    const long row = blockIdx.x;
    bf16 *xr = res + row * DIM;
    float v[8], wv[8];
    pdl_trigger();
    load8(w + c, wv);  // the norm weights are constant: read before the preceding kernel has finished
    pdl_wait();
    load8(xr + c, v);
    if (d) {
        float dv[8];
        load8(d + row * DIM + c, dv);
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = rbf(v[j] + dv[j]);
        store8(xr + c, v);
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) ss += v[j] * v[j];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < NW; k++) tot += red[k];
    const float r = rsqrtf(tot / DIM + eps);
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; j++) o[j] = rbf(v[j] * r) * wv[j];
    store8(out + row * DIM + c, o);
}

// out[r, c] = bf16(bf16(silu(gate)) * up) with gu = [gate | up] per row, F columns each (kernels/voxcpm.cu:92-99).
__global__ void __launch_bounds__(256) k_silu_mul(const bf16 *gu, bf16 *out, int rows, int F) {
    pdl_trigger();
    pdl_wait();
    const long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;  // vector index
    const int fv = F / 8;
    if (i >= static_cast<long>(rows) * fv) return;
    const long r = i / fv;
    const int c = static_cast<int>(i - r * fv) * 8;
    float g[8], u[8], o[8];
    load8(gu + r * 2 * F + c, g);
    load8(gu + r * 2 * F + F + c, u);
#pragma unroll
    for (int j = 0; j < 8; j++) o[j] = rbf(g[j] / (1.f + __expf(-g[j]))) * u[j];
    store8(out + r * F + c, o);
}

// In place over n elements (n % 8 == 0): op 0 = silu (kernels/voxcpm.cu:80-83); op 1 = FSQ,
// h = bf16(rint(bf16(bf16(tanh(h)) * scale)) / scale) (kernels/voxcpm.cu:370-375).
__global__ void __launch_bounds__(256) k_pointwise(bf16 *x, long n, int op, float scale) {
    pdl_trigger();
    pdl_wait();
    const long i = (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
    if (i >= n) return;
    float v[8];
    load8(x + i, v);
#pragma unroll
    for (int j = 0; j < 8; j++) {
        if (op == 0) {
            v[j] = v[j] / (1.f + __expf(-v[j]));
        } else {
            const float t = rbf(tanhf(v[j]));
            v[j] = rintf(rbf(t * scale)) / scale;
        }
    }
    store8(x + i, v);
}

// DiT input sequences [mu0, mu1, t, cond x4, x x4] for 2B rows (kernels/voxcpm.cu:299-315): rows < B carry
// mu = [B][2][H], rows >= B zeros (the unconditional branch); condp and xp are [B][4][H], shared by both halves.
// With seq == 5 and mu == null: the local encoder's [special, x0..x3] per patch (kernels/voxcpm.cu:325-331),
// `temb` then being the special token and rows = n patches.
__global__ void __launch_bounds__(256) k_build_seq(bf16 *seq_out, const bf16 *mu, const bf16 *temb,
                                                   const bf16 *condp, const bf16 *xp, int rows, int B, int seq,
                                                   int H) {
    const long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int hv = H / 8;
    if (i >= static_cast<long>(rows) * seq * hv) return;
    const int c = static_cast<int>(i % hv) * 8;
    const long rt = i / hv;
    const int tok = static_cast<int>(rt % seq);
    const int r = static_cast<int>(rt / seq);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (seq == 5) {
        v = tok == 0 ? *reinterpret_cast<const uint4 *>(temb + c)
                     : *reinterpret_cast<const uint4 *>(xp + (static_cast<long>(r) * 4 + tok - 1) * H + c);
    } else {
        const int s = r % B;
        if (tok < 2) {
            if (r < B) v = *reinterpret_cast<const uint4 *>(mu + (static_cast<long>(s) * 2 + tok) * H + c);
        } else if (tok == 2) {
            v = *reinterpret_cast<const uint4 *>(temb + c);
        } else if (tok < 7) {
            v = *reinterpret_cast<const uint4 *>(condp + (static_cast<long>(s) * 4 + tok - 3) * H + c);
        } else {
            v = *reinterpret_cast<const uint4 *>(xp + (static_cast<long>(s) * 4 + tok - 7) * H + c);
        }
    }
    *reinterpret_cast<uint4 *>(seq_out + rt * H + c) = v;
}

// Block-wide sum over 256 threads.
__device__ __forceinline__ float block_sum256(float v, float *red) {
    v = warp_sum(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; k++) t += red[k];
    return t;
}

// Classifier-free guidance (CFG-Zero*) and one Euler step for take s (block s, 256 threads = 4 frames x 64
// channels), the roundings of kernels/voxcpm.cu:334-345. The DiT output rows are read where they lie: frame t of
// row r at out[((r * seq + first + t) * 64 + c)], so the noisy-frame tokens need not be gathered first.
__global__ void __launch_bounds__(256) k_cfg_euler(bf16 *x, const bf16 *out, int B, int seq, int first, float dt,
                                                   float cfg) {
    __shared__ float red[8];
    const int s = blockIdx.x, i = threadIdx.x, t = i >> 6, c = i & 63;
    const float pos = bf2f(out[((static_cast<long>(s) * seq + first + t) << 6) + c]);
    const float neg = bf2f(out[((static_cast<long>(B + s) * seq + first + t) << 6) + c]);
    const float dot = rbf(block_sum256(rbf(pos * neg), red));
    const float nn = rbf(rbf(block_sum256(rbf(neg * neg), red)) + 1e-8f);
    const float st = rbf(dot / nn);
    const float a = rbf(neg * st);
    const float dv = rbf(a + rbf(cfg * rbf(pos - a)));
    const long xi = static_cast<long>(s) * 256 + i;
    x[xi] = f2bf(bf2f(x[xi]) - rbf(dt * dv));
}

// End of a decoding step (kernels/voxcpm.cu:415-433), one block: the new patch of every take goes to
// patches[s][n] (n = ctr[1] < max_steps), a take whose stop logits ask to stop after more than min_len patches
// records n, then ctr = [position + 1, n + 1] and, with per-take lengths, every lens[s] + 1.
__global__ void __launch_bounds__(256) k_step_end(const bf16 *stop_logits, const bf16 *patch, bf16 *patches,
                                                  int *stop, int *ctr, int *lens, int B, int min_len,
                                                  int max_steps) {
    const int n = ctr[1];
    if (n < max_steps) {
        for (int v = threadIdx.x; v < B * 32; v += blockDim.x) {
            const int s = v >> 5, e = (v & 31) * 8;
            *reinterpret_cast<uint4 *>(patches + (static_cast<long>(s) * max_steps + n) * 256 + e) =
                *reinterpret_cast<const uint4 *>(patch + static_cast<long>(s) * 256 + e);
        }
    }
    for (int s = threadIdx.x; s < B; s += blockDim.x) {
        const bool want = bf2f(stop_logits[2 * s + 1]) > bf2f(stop_logits[2 * s]);
        if (want && n > min_len && stop[s] < 0) stop[s] = n;
        if (lens) lens[s] += 1;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        ctr[0] += 1;
        ctr[1] = n + 1;
    }
}

// Condition of the decoding loop (Engine::decode, src/model.rs:784-793): one more step while fewer than max_steps
// patches exist (ctr[1]) and some take has not stopped (stop[s] < 0). One block; thread 0 sets the WHILE node's
// condition. status[0] counts the steps the loop ran in this launch (the first test, upstream of the WHILE node,
// resets it); the loop also ends after max_steps steps whatever ctr[1] says, with status[1] = 1, so a step that
// failed to advance ctr[1] cannot keep the device in the loop.
__global__ void __launch_bounds__(256) k_loop_test(cudaGraphConditionalHandle h, const int *stop, const int *ctr,
                                                   int *status, int B, int max_steps, int first) {
    int open = 0;
    for (int s = threadIdx.x; s < B; s += blockDim.x) open |= stop[s] < 0;
    open = __syncthreads_or(open);
    if (threadIdx.x == 0) {
        const int ran = first ? 0 : status[0] + 1;
        bool more = open && ctr[1] < max_steps;
        if (first) status[1] = 0;
        if (more && ran >= max_steps) {
            status[1] = 1;
            more = false;
        }
        status[0] = ran;
        cudaGraphSetConditional(h, more ? 1u : 0u);
    }
}

}  // namespace glue
