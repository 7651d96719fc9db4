// C ABI of the sm_100a attention hot path (declarations and reference citations in include/oumu_attn.h).
// Host side: argument validation, TMA tensor-map encoding, launch shapes. Nothing here allocates, synchronises
// or reads device memory (except oumu_device_error), so every entry point can be captured in a CUDA graph.
#include "../../include/oumu_attn.h"
#include "../../include/oumu_step.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "decode.cuh"
#include "feeders.cuh"
#include "full_small.cuh"
#include "gemm_tc.cuh"
#include "prefill_tc.cuh"
#include "prefill_pp.cuh"
#include "small_tc.cuh"
#include "step_glue.cuh"

namespace {

thread_local char g_last_cuda[256] = "";

int cuda_fail(cudaError_t e) {
    std::snprintf(g_last_cuda, sizeof(g_last_cuda), "%s", cudaGetErrorString(e));
    return OUMU_ERR_CUDA;
}
#define OUMU_CK(x)                                   \
    do {                                             \
        cudaError_t e_ = (x);                        \
        if (e_ != cudaSuccess) return cuda_fail(e_); \
    } while (0)

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

std::atomic<int> g_pdl{0};
std::atomic<int> g_drop_tile{0};  // oumu_test_drop_last_tile (off)

// Launch with programmatic stream serialization when oumu_set_pdl(1) is in effect.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = g_pdl.load(std::memory_order_relaxed) ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

constexpr int kMaxDevices = 64;
// Weight-streaming GEMM: pipeline depth per token tile (shared memory: stages x (16 KB + tile x 128 B) + the
// inbox). At 32 tokens, 8 stages keep 160 KB of weights in flight per SM: a GEMM whose tiles occupy only part of the
// SMs (gate|up on 96) still streams at the HBM rate (captured decoding step: 4.69 -> 4.55 ms against 4 stages).
constexpr int kGemmStages32 = 8, kGemmStages64 = 4, kGemmStages128 = 3;
constexpr int kPrefillPairMinSeq = 4096;  // sequences from this length take the ping-pong prefill kernel

constexpr int kSmemMax = 227 * 1024;

struct DevInfo {
    bool ready = false;
    int sms = 0;
};
DevInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

// SM count of the current device; first use on a device also raises the dynamic shared-memory limit of the
// kernels that need more than 48 KB.
int current_device(int *sms) {
    int d = 0;
    OUMU_CK(cudaGetDevice(&d));
    if (d < 0 || d >= kMaxDevices) return OUMU_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lk(g_dev_mu);
    DevInfo &di = g_dev[d];
    if (!di.ready) {
        OUMU_CK(cudaDeviceGetAttribute(&di.sms, cudaDevAttrMultiProcessorCount, d));
        OUMU_CK(cudaFuncSetAttribute(dec::k_attn_decode<128, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemMax));
        OUMU_CK(cudaFuncSetAttribute(dec::k_attn_decode<64, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemMax));
        OUMU_CK(cudaFuncSetAttribute(dec::k_attn_decode<128, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemMax));
        OUMU_CK(cudaFuncSetAttribute(dec::k_attn_decode<64, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemMax));
        OUMU_CK(cudaFuncSetAttribute(dec::k_attn_decode<128, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemMax));
        OUMU_CK(cudaFuncSetAttribute(dec::k_attn_decode<64, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemMax));
        OUMU_CK(cudaFuncSetAttribute(dec::k_attn_decode<128, true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemMax));
        OUMU_CK(cudaFuncSetAttribute(dec::k_attn_decode<64, true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemMax));
        OUMU_CK(cudaFuncSetAttribute(pp::k_attn_prefill_pp<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemMax));
        OUMU_CK(cudaFuncSetAttribute(pp::k_attn_prefill_pp<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemMax));
        OUMU_CK(cudaFuncSetAttribute(pf::k_attn_prefill<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     pf::Cfg<128>::SMEM));
        OUMU_CK(cudaFuncSetAttribute(pf::k_attn_prefill<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     pf::Cfg<64>::SMEM));
        OUMU_CK(cudaFuncSetAttribute(fs::k_attn_small_grp<128, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     fs::GCfg<128>::smem_bytes(fs::MAXM / fs::ROWS)));
        OUMU_CK(cudaFuncSetAttribute(fs::k_attn_small_grp<128, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     fs::GCfg<128>::smem_bytes(fs::MAXM / fs::ROWS)));
        OUMU_CK(cudaFuncSetAttribute(fs::k_attn_small_grp<64, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     fs::GCfg<64>::smem_bytes(fs::MAXM / fs::ROWS)));
        OUMU_CK(cudaFuncSetAttribute(fs::k_attn_small_grp<64, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     fs::GCfg<64>::smem_bytes(fs::MAXM / fs::ROWS)));
        OUMU_CK(cudaFuncSetAttribute(sq::k_attn_small_tc<128, 16, 3, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemMax));
        OUMU_CK(cudaFuncSetAttribute(sq::k_attn_small_tc<128, 16, 3, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemMax));
        OUMU_CK(cudaFuncSetAttribute(sq::k_attn_small_tc<64, 16, 3, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemMax));
        OUMU_CK(cudaFuncSetAttribute(sq::k_attn_small_tc<64, 16, 3, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemMax));
        OUMU_CK(cudaFuncSetAttribute(sq::k_attn_small_tc<128, 128, 2, false>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax));
        OUMU_CK(cudaFuncSetAttribute(sq::k_attn_small_tc<64, 128, 2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemMax));
        OUMU_CK(cudaFuncSetAttribute(gm::k_gemm<32, kGemmStages32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemMax));
        OUMU_CK(cudaFuncSetAttribute(gm::k_gemm<64, kGemmStages64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemMax));
        OUMU_CK(cudaFuncSetAttribute(gm::k_gemm<128, kGemmStages128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemMax));
        di.ready = true;
    }
    *sms = di.sms;
    return OUMU_OK;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link-time libcuda dependency).
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 2-D bf16 map over [outer][inner] (row pitch row_bytes) with a (box_inner x box_outer) box, 128-byte swizzle.
int make_map(CUtensorMap *m, const void *base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
             uint32_t box_inner, uint32_t box_outer) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) {
        std::snprintf(g_last_cuda, sizeof(g_last_cuda), "cuTensorMapEncodeTiled unavailable");
        return OUMU_ERR_CUDA;
    }
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        std::snprintf(g_last_cuda, sizeof(g_last_cuda), "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
        return OUMU_ERR_CUDA;
    }
    return OUMU_OK;
}

// 3-D bf16 map over the layer caches [slots][nk][maxlen][hd] restricted to the first T positions: dims
// {hd, T, slots * nk}, box {64, box_rows, 1}, 128-byte swizzle; boxes reaching past position T are clipped.
int make_map_cache(CUtensorMap *m, const void *base, int hd, int T, int planes, int maxlen, uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) {
        std::snprintf(g_last_cuda, sizeof(g_last_cuda), "cuTensorMapEncodeTiled unavailable");
        return OUMU_ERR_CUDA;
    }
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(hd), static_cast<cuuint64_t>(T), static_cast<cuuint64_t>(planes)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(hd) * 2, static_cast<cuuint64_t>(maxlen) * hd * 2};
    cuuint32_t box[3] = {64, box_rows, 1};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        std::snprintf(g_last_cuda, sizeof(g_last_cuda), "cuTensorMapEncodeTiled (cache) failed (%d)",
                      static_cast<int>(r));
        return OUMU_ERR_CUDA;
    }
    return OUMU_OK;
}

// 3-D bf16 map over a [rows][heads][hd] buffer with row pitch row_bytes, box {64, bh, br}, 128-byte swizzle: a box
// is br rows x bh heads x 64 columns, landing as bh * br rows of 128 bytes (row r, head h -> r * bh + h).
int make_map_heads(CUtensorMap *m, const void *base, int hd, int heads, int rows, uint64_t row_bytes, uint32_t bh,
                   uint32_t br) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) {
        std::snprintf(g_last_cuda, sizeof(g_last_cuda), "cuTensorMapEncodeTiled unavailable");
        return OUMU_ERR_CUDA;
    }
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(hd), static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(hd) * 2, row_bytes};
    cuuint32_t box[3] = {64, bh, br};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        std::snprintf(g_last_cuda, sizeof(g_last_cuda), "cuTensorMapEncodeTiled (heads) failed (%d)",
                      static_cast<int>(r));
        return OUMU_ERR_CUDA;
    }
    return OUMU_OK;
}

uint16_t f2b_host(float x) {  // round-to-nearest-even, NaN -> 0x7fc0 (src/gpu.rs:72-78)
    if (std::isnan(x)) return 0x7fc0;
    uint32_t u;
    std::memcpy(&u, &x, 4);
    return static_cast<uint16_t>((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}
float rb_host(float x) {
    uint32_t u = static_cast<uint32_t>(f2b_host(x)) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

bool head_dim_ok(int hd) { return hd == 64 || hd == 128; }

size_t decode_counter_bytes(int B, int nk) { return (static_cast<size_t>(B) * nk * 4 + 255) & ~static_cast<size_t>(255); }
size_t decode_part_bytes(int hd) {
    return 2 * static_cast<size_t>(hd == 128 ? dec::Cfg<128>::PART_FLOATS : dec::Cfg<64>::PART_FLOATS) * 4;
}

template <int HD, bool FUSED>
int launch_decode(const void *qkv, const void *kc, const void *vc, void *out, void *ws, size_t ws_bytes,
                  const int *pos, const int *lens, const float *cos_t, const float *sin_t, int B, int nq, int nk,
                  int maxlen, float scale, int sms, cudaStream_t st) {
    using C = dec::Cfg<HD>;
    const long tiles_max = static_cast<long>(B) * nk * ((maxlen + dec::TILE - 1) / dec::TILE);
    const size_t cbytes = decode_counter_bytes(B, nk), pbytes = decode_part_bytes(HD);
    if (ws_bytes < cbytes + pbytes) return OUMU_ERR_WORKSPACE;
    long grid = sms;
    if (grid > tiles_max) grid = tiles_max;
    const long fit = static_cast<long>((ws_bytes - cbytes) / pbytes);
    if (grid > fit) grid = fit;
    // shared memory: one stage per consumer warp, plus 1 KB to align the base to 1024 B
    const dec::Smem<HD> lay{B};
    if (lay.bytes() + 1024 > kSmemMax) return OUMU_ERR_UNSUPPORTED;
    const int smem = lay.bytes() + 1024;
    CUtensorMap tk, tv;
    const uint64_t rows = static_cast<uint64_t>(B) * nk * maxlen;
    int rc = make_map(&tk, kc, HD, rows, HD * 2, 64, dec::TILE);
    if (rc) return rc;
    rc = make_map(&tv, vc, HD, rows, HD * 2, 64, dec::TILE);
    if (rc) return rc;
    dec::Params P;
    P.qkv = static_cast<bf16 *>(const_cast<void *>(qkv));
    P.kc = static_cast<bf16 *>(const_cast<void *>(kc));
    P.vc = static_cast<bf16 *>(const_cast<void *>(vc));
    P.cos_t = cos_t;
    P.sin_t = sin_t;
    P.out = static_cast<bf16 *>(out);
    P.cnt = static_cast<int *>(ws);
    P.part = reinterpret_cast<float *>(static_cast<char *>(ws) + cbytes);
    P.pos = pos;
    P.lens = lens;
    P.B = B;
    P.nq = nq;
    P.nk = nk;
    P.maxlen = maxlen;
    P.sl2 = scale * 1.4426950408889634f;
    // the fault-injection build only while oumu_test_drop_last_tile is on
    OUMU_CK(launch_k(g_drop_tile.load(std::memory_order_relaxed) ? dec::k_attn_decode<HD, FUSED, true>
                                                                  : dec::k_attn_decode<HD, FUSED, false>,
                     dim3(static_cast<unsigned>(grid)), dim3(dec::NTHREADS), smem, st, tk, tv, P));
    return OUMU_OK;
}

template <int HD>
int launch_small(const void *qkv, void *out, int rows, int seq, int causal, int nq, int nk, float scale, int sms,
                 cudaStream_t st, const float *cos_t = nullptr, const float *sin_t = nullptr) {
    const int G = nq / nk;
    if (G > 1 && G * seq <= fs::MAXM) {  // grouped heads: one CTA per (sequence, kv head), K/V staged once
        const long ctas = static_cast<long>(rows / seq) * nk;
        if (ctas > 0x7fffffffL) return OUMU_ERR_UNSUPPORTED;
        const int mt = (G * seq + fs::ROWS - 1) / fs::ROWS;
        auto kern = cos_t ? fs::k_attn_small_grp<HD, true> : fs::k_attn_small_grp<HD, false>;
        kern<<<static_cast<unsigned>(ctas), mt * 32, fs::GCfg<HD>::smem_bytes(mt), st>>>(
            static_cast<const bf16 *>(qkv), static_cast<bf16 *>(out), seq, causal, nq, nk,
            scale * 1.4426950408889634f, cos_t, sin_t);
        OUMU_CK(cudaGetLastError());
        return OUMU_OK;
    }
    if (cos_t) return OUMU_ERR_UNSUPPORTED;  // rope fused only into the grouped kernel
    const long units = static_cast<long>(rows / seq) * nq;
    long grid = (units + fs::WARPS - 1) / fs::WARPS;
    const long cap = static_cast<long>(sms) * 8;
    if (grid > cap) grid = cap;
    const int smem = fs::WARPS * fs::Cfg<HD>::WARP_BYTES;
    fs::k_attn_small<HD><<<static_cast<int>(grid), fs::WARPS * 32, smem, st>>>(
        static_cast<const bf16 *>(qkv), static_cast<bf16 *>(out), rows / seq, seq, causal, nq, nk,
        scale * 1.4426950408889634f);
    OUMU_CK(cudaGetLastError());
    return OUMU_OK;
}

// q heads per unit of the tensor-core short-sequence kernel: the largest divisor of the group (grouped heads) or of
// nq (one q head per kv head, at most 8 stacked) with at most 128 stacked query rows.
int small_tc_heads(int seq, int nq, int nk) {
    const int G = nq / nk, top = G > 1 ? G : (nq < 8 ? nq : 8), of = G > 1 ? G : nq;
    for (int d = top; d >= 1; d--)
        if (of % d == 0 && d * seq <= 128) return d;
    return 1;
}

// The persistent tensor-core kernel streams its units through a pipeline that takes ~5 us to fill and drain; with
// fewer than 4 units per SM (the local encoder's 5-token calls, small batches) the one-CTA-per-unit kernel finishes
// first, and for one q head per kv head (no group to stack) it is faster at every size measured.
bool small_use_tc(int rows, int seq, int nq, int nk, int sms) {
    const int G = nq / nk;
    if (G < 2) return false;
    const long units = static_cast<long>(rows / seq) * nk * (G / small_tc_heads(seq, nq, nk));
    return units >= 4L * sms;
}

// Short sequences (seq <= 16) on the tensor cores (sq::k_attn_small_tc): the unit shape, the slots, the maps.
template <int HD>
int launch_small_tc(const void *qkv, void *out, int rows, int seq, int causal, int nq, int nk, float scale, int sms,
                    cudaStream_t st, const float *cos_t = nullptr, const float *sin_t = nullptr) {
    const int G = nq / nk;
    const int HS = small_tc_heads(seq, nq, nk);
    const int KS = G > 1 ? 1 : HS;
    if (cos_t && KS != 1) return OUMU_ERR_UNSUPPORTED;  // rope fused only with grouped heads
    sq::Params P;
    P.cos_t = cos_t;
    P.sin_t = sin_t;
    P.seq = seq;
    P.causal = causal ? 1 : 0;
    P.nq = nq;
    P.nk = nk;
    P.G = G;
    P.HS = HS;
    P.KS = KS;
    P.qrows = HS * seq;
    P.krows = KS * seq;
    P.ns = (P.krows + 15) / 16 * 16;
    P.ups = G > 1 ? nk * (G / HS) : nq / HS;
    const long units = static_cast<long>(rows / seq) * P.ups;
    if (units > 0x7fffffffL) return OUMU_ERR_UNSUPPORTED;
    P.units = static_cast<int>(units);
    constexpr int NBOX = HD / 64;
    P.qbox = (P.qrows * 128 + 1023) / 1024 * 1024;
    P.kbox = P.ns * 128;
    P.slot = NBOX * (P.qbox + 2 * P.kbox);
    const int room = kSmemMax - sq::smem_bytes(0, 0);
    P.nslot = room / P.slot < sq::NSLOT_MAX ? room / P.slot : sq::NSLOT_MAX;
    if (P.nslot < 2) return OUMU_ERR_UNSUPPORTED;
    P.sl2 = scale * 1.4426950408889634f;
    const uint64_t wq = static_cast<uint64_t>(nq + 2 * nk) * HD * 2;
    CUtensorMap tq, tkv, tout;
    int rc = make_map_heads(&tq, qkv, HD, nq + 2 * nk, rows, wq, HS, seq);
    if (rc) return rc;
    rc = make_map_heads(&tkv, qkv, HD, nq + 2 * nk, rows, wq, KS, seq);
    if (rc) return rc;
    rc = make_map_heads(&tout, out, HD, nq, rows, static_cast<uint64_t>(nq) * HD * 2, HS, seq);
    if (rc) return rc;
    const int grid = P.units < sms ? P.units : sms;
    // more than half an SM's shared memory, so that no two CTAs (each allocating all 512 TMEM columns) share an SM
    const int smem = std::max(sq::smem_bytes(P.slot, P.nslot), 120 * 1024);
    if (KS == 1) {
        auto kern = cos_t ? sq::k_attn_small_tc<HD, 16, 3, true> : sq::k_attn_small_tc<HD, 16, 3, false>;
        OUMU_CK(launch_k(kern, dim3(grid), dim3(sq::nthreads(3)), smem, st, tq, tkv, tout, P));
    } else {
        OUMU_CK(launch_k(sq::k_attn_small_tc<HD, 128, 2, false>, dim3(grid), dim3(sq::nthreads(2)), smem, st, tq,
                         tkv, tout, P));
    }
    return OUMU_OK;
}

// The plan of the prefill's KV epilogue (pf::CopyPlan). It applies to one causal sequence whose grid plus one copy
// CTA per q head fits on the SMs at once; it is the same for every q head. A q head's slots are cut into at most
// PLAN_GROUPS groups. Each key tile t hands its groups, kPfLoopBytes of stores at a time, to the query tiles that
// load tile t for their attention and not as their last tile (qt > t), shortest first, but never to the two longest
// query tiles, which bound the kernel: those stores run while the CTA computes. The groups left go one by one to
// whichever CTA that does not load the tile is expected to be free first: query tile qt is busy until ~kPfFixedUs + (qt + 1) * kPfTileUs, the copy CTA from kPfCopyStartUs, and each
// group costs its stores at kPfStoreGBs per SM, plus a load of the tile for the first group a CTA takes of it.
constexpr double kPfFixedUs = 5.0, kPfTileUs = 1.6, kPfCopyStartUs = 1.5, kPfLoadUs = 0.5;
constexpr double kPfStoreGBs = 85.0, kPfLoopBytes = 384.0 * 1024;

pf::CopyPlan prefill_copy_plan(int hd, int seq, int causal, int nq, int nk, int nseq, int slots, int sms) {
    pf::CopyPlan plan;
    std::memset(&plan, 0, sizeof(plan));
    const int qtiles = (seq + pf::BM - 1) / pf::BM, G = nq / nk;
    if (slots <= 0 || !causal || nseq != 1 || qtiles > pf::PLAN_MAX || qtiles < 2 ||
        static_cast<long>(nq) * (qtiles + 1) > sms)
        return plan;
    const int per = (slots + G - 1) / G;  // slots per q head (the widest share)
    int ngroups = std::min(per, pf::PLAN_GROUPS);
    plan.gs = (per + ngroups - 1) / ngroups;
    ngroups = (per + plan.gs - 1) / plan.gs;
    plan.planned = 1;
    for (int t = 0; t < pf::PLAN_MAX; t++)
        for (int sg = 0; sg < pf::PLAN_GROUPS; sg++) plan.owner[t][sg] = -1;
    const double item_bytes = static_cast<double>(plan.gs) * 2 * pf::BN * hd * 2;
    const double item_us = item_bytes / (kPfStoreGBs * 1e3);
    const int loop_cap = std::max(1, static_cast<int>(kPfLoopBytes / item_bytes));
    double busy[pf::PLAN_MAX + 1];
    for (int q = 0; q < qtiles; q++) busy[q] = kPfFixedUs + (q + 1) * kPfTileUs;
    busy[qtiles] = kPfCopyStartUs;
    for (int t = 0; t < qtiles; t++) {
        int sg = 0;
        for (int q = t + 1; q < qtiles - 2 && sg < ngroups; q++)
            for (int k = 0; k < loop_cap && sg < ngroups; k++) plan.owner[t][sg++] = static_cast<signed char>(q);
        bool loaded[pf::PLAN_MAX + 1] = {};
        for (; sg < ngroups; sg++) {
            int best = qtiles;
            double bt = busy[qtiles] + (loaded[qtiles] ? 0.0 : kPfLoadUs);
            for (int q = 0; q < t; q++) {
                const double c = busy[q] + (loaded[q] ? 0.0 : kPfLoadUs);
                if (c < bt) {
                    bt = c;
                    best = q;
                }
            }
            plan.owner[t][sg] = static_cast<signed char>(best);
            busy[best] = bt + item_us;
            loaded[best] = true;
        }
    }
    return plan;
}

// Prefill attention; with kc/vc (slots > 0) also the KV epilogue into every slot's first `seq` positions.
template <int HD>
int launch_prefill(const void *qkv, void *out, int rows, int seq, int causal, int nq, int nk, float scale,
                   cudaStream_t st, void *kc = nullptr, void *vc = nullptr, int slots = 0, int maxlen = 0) {
    CUtensorMap tm, tkc, tvc;
    std::memset(&tkc, 0, sizeof(tkc));
    std::memset(&tvc, 0, sizeof(tvc));
    const uint64_t width = static_cast<uint64_t>(nq + 2 * nk) * HD;
    int rc = make_map(&tm, qkv, width, rows, width * 2, 64, pf::BM);
    if (rc) return rc;
    if (slots > 0) {
        rc = make_map_cache(&tkc, kc, HD, seq, slots * nk, maxlen, pf::BN);
        if (rc) return rc;
        rc = make_map_cache(&tvc, vc, HD, seq, slots * nk, maxlen, pf::BN);
        if (rc) return rc;
    }
    const int nseq = rows / seq, qtiles = (seq + pf::BM - 1) / pf::BM;
    if (nseq > 65535 || qtiles > 65535) return OUMU_ERR_UNSUPPORTED;
    int sms = 0;
    int rc2 = current_device(&sms);
    if (rc2) return rc2;
    // Long sequences without the KV epilogue: two query tiles per CTA in ping-pong (pp::k_attn_prefill_pp), whose
    // output is bit-identical. Measured on a B200 (16 q / 2 kv heads, hd 128, causal): T = 4096 92 against 99 us,
    // T = 16384 1.31 against 1.43 ms; at T = 2048 the pairs' causal chains on half as many CTAs lose (50 against
    // 31 us).
    if (slots == 0 && seq >= kPrefillPairMinSeq) {
        const int pairs = (qtiles + 1) / 2;
        // more than half an SM's shared memory, so that no two CTAs (each allocating all 512 TMEM columns) share an SM
        const int smem = std::max(pp::Cfg<HD>::SMEM, 120 * 1024);
        OUMU_CK(launch_k(pp::k_attn_prefill_pp<HD>, dim3(nq, pairs, nseq), dim3(pp::NTHREADS), smem, st,
                         tm, static_cast<bf16 *>(out), seq, causal, nq, nk, scale * 1.4426950408889634f));
        return OUMU_OK;
    }
    const pf::CopyPlan plan = prefill_copy_plan(HD, seq, causal, nq, nk, nseq, slots, sms);
    dim3 grid(nq, qtiles + (plan.planned ? 1 : 0), nseq);
    OUMU_CK(launch_k(pf::k_attn_prefill<HD>, grid, dim3(pf::NTHREADS), pf::Cfg<HD>::SMEM, st, tm,
                     static_cast<bf16 *>(out), seq, causal, nq, nk, scale * 1.4426950408889634f, tkc, tvc, slots,
                     plan));
    return OUMU_OK;
}

// Token tile of the GEMM for M tokens, the tile counts and the K split (CTAs per output tile = the cluster size).
struct GemmShape {
    int tn, tt, nt, kb, split;
    long tiles;
};

GemmShape gemm_shape(int M, int N, int K) {
    GemmShape g;
    g.tn = M <= 32 ? 32 : (M <= 64 ? 64 : 128);
    g.tt = (M + g.tn - 1) / g.tn;
    g.nt = (N + gm::BW - 1) / gm::BW;
    g.kb = K / gm::BK;
    g.tiles = static_cast<long>(g.tt) * g.nt;
    g.split = 1;
    return g;
}

// Clusters of `split` CTAs of k_gemm<TN, STAGES> resident at once on the current device (occupancy query, cached
// per device and split; 0 if the query fails). A kernel that allocates TMEM runs one CTA per SM.
template <int TN, int STAGES>
int gemm_capacity(int dev, int split) {
    static int cache[kMaxDevices][gm::MAX_SPLIT + 1];
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    int &c = cache[dev][split];
    if (c == 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>(split * 1024));
        cfg.blockDim = dim3(gm::NTHREADS);
        cfg.dynamicSmemBytes = gm::Cfg<TN, STAGES>::smem_bytes(split);
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = static_cast<unsigned>(split);
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, reinterpret_cast<const void *>(gm::k_gemm<TN, STAGES>), &cfg) !=
            cudaSuccess) {
            cudaGetLastError();
            n = -1;
        }
        c = n;
    }
    return c > 0 ? c : 0;
}

// The largest split (at most 8, at most one per K block) whose grid is resident in one wave; 1 when even that
// does not fit (many tiles: the DiT's token counts).
template <int TN, int STAGES>
void gemm_pick_split(GemmShape &g, int dev) {
    g.split = 1;
    const int hi = g.kb < gm::MAX_SPLIT ? g.kb : gm::MAX_SPLIT;
    for (int sp = hi; sp >= 2; sp--) {
        if (g.tiles <= gemm_capacity<TN, STAGES>(dev, sp)) {
            g.split = sp;
            return;
        }
    }
}

bool gemm_args_ok(const void *x, int ldx, const void *w, const void *y, int ldy, int M, int N, int K) {
    return x && w && y && M >= 1 && N >= 1 && K >= gm::BK && K % gm::BK == 0 && ldx >= K && ldx % 8 == 0 &&
           ldy >= N && aligned16(x) && aligned16(w);
}

template <int TN, int STAGES>
int launch_gemm(const void *x, int ldx, const void *w, void *y, int ldy, const void *bias, int M, int N, int K,
                GemmShape gs, int dev, cudaStream_t st, int act = 0) {
    // the SwiGLU form takes the split the plain form would (so it sums each output in the same order and its gate
    // and up values are those the plain form stores); its inbox may be larger, which only matters for residency
    gemm_pick_split<TN, STAGES>(gs, dev);
    if (gs.tiles * gs.split > 0x7fffffffL || gm::Cfg<TN, STAGES>::smem_bytes(gs.split, act) > kSmemMax)
        return OUMU_ERR_UNSUPPORTED;
    CUtensorMap tw, tx;
    int rc = make_map(&tw, w, K, N, static_cast<uint64_t>(K) * 2, gm::BK, gm::BW);
    if (rc) return rc;
    rc = make_map(&tx, x, K, M, static_cast<uint64_t>(ldx) * 2, gm::BK, TN);
    if (rc) return rc;
    gm::Params P;
    P.y = static_cast<bf16 *>(y);
    P.bias = static_cast<const bf16 *>(bias);
    P.ldy = ldy;
    P.M = M;
    P.N = N;
    P.NT = gs.nt;
    P.KB = gs.kb;
    P.split = gs.split;
    P.act = act;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(gs.tiles * gs.split));
    cfg.blockDim = dim3(gm::NTHREADS);
    cfg.dynamicSmemBytes = gm::Cfg<TN, STAGES>::smem_bytes(gs.split, act);
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(gs.split);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = g_pdl.load(std::memory_order_relaxed) ? 2 : 1;
    OUMU_CK(cudaLaunchKernelEx(&cfg, gm::k_gemm<TN, STAGES>, tw, tx, P));
    return OUMU_OK;
}

}  // namespace

extern "C" {

const char *oumu_status_string(int s) {
    switch (s) {
        case OUMU_OK: return "ok";
        case OUMU_ERR_INVALID: return "invalid argument";
        case OUMU_ERR_UNSUPPORTED: return "unsupported shape";
        case OUMU_ERR_WORKSPACE: return "workspace too small";
        case OUMU_ERR_CUDA: return "CUDA error";
        case OUMU_ERR_DEVICE: return "device-side error";
        default: return "unknown status";
    }
}

const char *oumu_last_cuda_error(void) { return g_last_cuda; }

int oumu_set_pdl(int enable) { return g_pdl.exchange(enable ? 1 : 0); }

int oumu_rotary_tables(int maxlen, int hd, const double *ext, float *cos_out, float *sin_out) {
    if (maxlen < 1 || hd < 2 || (hd & 1) || !cos_out || !sin_out) return OUMU_ERR_INVALID;
    const int half = hd / 2;
    for (int p = 0; p < maxlen; p++)
        for (int i = 0; i < half; i++) {
            const float inv = 1.0f / powf(10000.0f, static_cast<float>(2 * i) / static_cast<float>(hd));
            const float e = ext ? static_cast<float>(ext[i]) : 1.0f;
            const float fr = (static_cast<float>(p) * (1.0f / e)) * inv;
            cos_out[static_cast<long>(p) * half + i] = rb_host(cosf(fr));
            sin_out[static_cast<long>(p) * half + i] = rb_host(sinf(fr));
        }
    return OUMU_OK;
}

int oumu_rope(void *qkv, const float *cos_t, const float *sin_t, const int *pos, int rows, int seq, int nq, int nk,
              int hd, oumu_stream_t stream) {
    if (!qkv || !cos_t || !sin_t || rows < 0 || seq < 0 || nq < 1 || nk < 0) return OUMU_ERR_INVALID;
    if (seq == 0 && !pos) return OUMU_ERR_INVALID;
    if (!head_dim_ok(hd)) return OUMU_ERR_UNSUPPORTED;
    if (!aligned16(qkv) || !aligned16(cos_t) || !aligned16(sin_t)) return OUMU_ERR_INVALID;
    if (rows == 0) return OUMU_OK;
    const long total = static_cast<long>(rows) * (nq + nk) * (hd / 16);
    k_rope<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(static_cast<bf16 *>(qkv), cos_t, sin_t, pos,
                                                                        rows, seq, nq, nk, hd);
    OUMU_CK(cudaGetLastError());
    return OUMU_OK;
}

int oumu_kv_write(const void *qkv, void *kc, void *vc, const int *pos, int slots, int rows, int nq, int nk, int hd,
                  int maxlen, oumu_stream_t stream) {
    if (!qkv || !kc || !vc || slots < 0 || rows < 0 || nq < 0 || nk < 1 || maxlen < 1) return OUMU_ERR_INVALID;
    if (!head_dim_ok(hd)) return OUMU_ERR_UNSUPPORTED;
    if (!aligned16(qkv) || !aligned16(kc) || !aligned16(vc)) return OUMU_ERR_INVALID;
    if (!pos && rows > maxlen) return OUMU_ERR_INVALID;
    const long total = static_cast<long>(slots) * rows * nk * (hd / 8) * 2;
    if (total == 0) return OUMU_OK;
    k_kv_write<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(
        static_cast<const bf16 *>(qkv), static_cast<bf16 *>(kc), static_cast<bf16 *>(vc), pos, slots, rows, nq, nk,
        hd, maxlen);
    OUMU_CK(cudaGetLastError());
    return OUMU_OK;
}

int oumu_decode_prologue(void *qkv, void *kc, void *vc, const float *cos_t, const float *sin_t, const int *pos,
                         const int *lens, int B, int nq, int nk, int hd, int maxlen, oumu_stream_t stream) {
    if (!qkv || !kc || !vc || (!pos && !lens) || B < 0 || nq < 1 || nk < 1 || maxlen < 1) return OUMU_ERR_INVALID;
    if ((cos_t == nullptr) != (sin_t == nullptr)) return OUMU_ERR_INVALID;
    if (!head_dim_ok(hd)) return OUMU_ERR_UNSUPPORTED;
    if (!aligned16(qkv) || !aligned16(kc) || !aligned16(vc) || (cos_t && (!aligned16(cos_t) || !aligned16(sin_t))))
        return OUMU_ERR_INVALID;
    if (B == 0) return OUMU_OK;
    OUMU_CK(launch_k(k_decode_prologue, dim3(B), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream),
                     static_cast<bf16 *>(qkv), static_cast<bf16 *>(kc), static_cast<bf16 *>(vc), cos_t, sin_t, pos,
                     lens, nq, nk, hd, maxlen));
    return OUMU_OK;
}

size_t oumu_attn_decode_workspace(int B, int nq, int nk, int hd, int maxlen) {
    if (B < 1 || nk < 1 || nq % nk || !head_dim_ok(hd) || maxlen < 1) return 0;
    int sms = 0;
    if (current_device(&sms) != OUMU_OK) sms = 160;
    const long tiles_max = static_cast<long>(B) * nk * ((maxlen + dec::TILE - 1) / dec::TILE);
    const long grid = tiles_max < sms ? tiles_max : sms;
    return decode_counter_bytes(B, nk) + static_cast<size_t>(grid) * decode_part_bytes(hd);
}

int oumu_attn_decode_reset(void *workspace, size_t workspace_bytes, int B, int nq, int nk, int hd, int maxlen,
                           oumu_stream_t stream) {
    (void)nq;
    (void)hd;
    (void)maxlen;
    if (!workspace || B < 1 || nk < 1) return OUMU_ERR_INVALID;
    const size_t cb = decode_counter_bytes(B, nk);
    if (workspace_bytes < cb) return OUMU_ERR_WORKSPACE;
    OUMU_CK(cudaMemsetAsync(workspace, 0, cb, stream));
    return OUMU_OK;
}

namespace {
// Every argument check of the decode entry points except the workspace's, in one place: a call that fails any of
// them has launched and queued nothing.
int decode_check(const void *qkv, const void *kc, const void *vc, const void *out, const float *cos_t,
                 const float *sin_t, const int *pos, const int *lens, int B, int nq, int nk, int hd, int maxlen,
                 float scale) {
    if (!qkv || !kc || !vc || !out || (!pos && !lens)) return OUMU_ERR_INVALID;
    if (B < 1 || nq < 1 || nk < 1 || nq % nk || maxlen < 1 || !(scale > 0.f)) return OUMU_ERR_INVALID;
    if ((cos_t == nullptr) != (sin_t == nullptr)) return OUMU_ERR_INVALID;
    if (!head_dim_ok(hd) || nq / nk > dec::GMAX || B > 4096) return OUMU_ERR_UNSUPPORTED;
    if (static_cast<long>(B) * nk * maxlen >= (1L << 31)) return OUMU_ERR_UNSUPPORTED;
    // the per-take length table and tile prefix live in shared memory beside the stages
    const int lay = hd == 128 ? dec::Smem<128>{B}.bytes() : dec::Smem<64>{B}.bytes();
    if (lay + 1024 > kSmemMax) return OUMU_ERR_UNSUPPORTED;
    if (!aligned16(qkv) || !aligned16(kc) || !aligned16(vc) || !aligned16(out) ||
        (cos_t && (!aligned16(cos_t) || !aligned16(sin_t))))
        return OUMU_ERR_INVALID;
    return OUMU_OK;
}

// Launch of a decode whose arguments passed decode_check.
int decode_launch(bool fused, const void *qkv, const void *kc, const void *vc, void *out, void *workspace,
                  size_t workspace_bytes, const float *cos_t, const float *sin_t, const int *pos, const int *lens,
                  int B, int nq, int nk, int hd, int maxlen, float scale, cudaStream_t st) {
    int sms = 0;
    int rc = current_device(&sms);
    if (rc) return rc;
    if (fused)
        return hd == 128 ? launch_decode<128, true>(qkv, kc, vc, out, workspace, workspace_bytes, pos, lens, cos_t,
                                                    sin_t, B, nq, nk, maxlen, scale, sms, st)
                         : launch_decode<64, true>(qkv, kc, vc, out, workspace, workspace_bytes, pos, lens, cos_t,
                                                   sin_t, B, nq, nk, maxlen, scale, sms, st);
    return hd == 128 ? launch_decode<128, false>(qkv, kc, vc, out, workspace, workspace_bytes, pos, lens, nullptr,
                                                 nullptr, B, nq, nk, maxlen, scale, sms, st)
                     : launch_decode<64, false>(qkv, kc, vc, out, workspace, workspace_bytes, pos, lens, nullptr,
                                                nullptr, B, nq, nk, maxlen, scale, sms, st);
}

int decode_entry(bool fused, const void *qkv, const void *kc, const void *vc, void *out, void *workspace,
                 size_t workspace_bytes, const float *cos_t, const float *sin_t, const int *pos, const int *lens, int B,
                 int nq, int nk, int hd, int maxlen, float scale, oumu_stream_t stream) {
    int rc = decode_check(qkv, kc, vc, out, cos_t, sin_t, pos, lens, B, nq, nk, hd, maxlen, scale);
    if (rc) return rc;
    if (!workspace || !aligned16(workspace)) return OUMU_ERR_INVALID;
    return decode_launch(fused, qkv, kc, vc, out, workspace, workspace_bytes, cos_t, sin_t, pos, lens, B, nq, nk, hd,
                         maxlen, scale, reinterpret_cast<cudaStream_t>(stream));
}
}  // namespace

int oumu_attn_decode(const void *qkv, const void *kc, const void *vc, void *out, void *workspace,
                     size_t workspace_bytes, const int *pos, const int *lens, int B, int nq, int nk, int hd,
                     int maxlen, float scale, oumu_stream_t stream) {
    return decode_entry(false, qkv, kc, vc, out, workspace, workspace_bytes, nullptr, nullptr, pos, lens, B, nq, nk,
                        hd, maxlen, scale, stream);
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------------------
// Decode attention without a caller-supplied workspace.
//
// Some hosts cannot hand this library device memory for scratch: a plug-in that receives only its input and output
// buffers from an engine that owns every device allocation, or a host whose memory policy forbids a library to
// allocate on its own (and whose workspace plan has no room for this kernel's scratch). For them the split-KV
// partials and the combine counters live in this file-scope array instead: every device that loads the library
// keeps its own copy, OUMU_DECODE_STATIC_SCRATCH_BYTES large, until the process exits.
// ------------------------------------------------------------------------------------------------------------
static __device__ __align__(256) unsigned char oumu_decode_static_scratch[OUMU_DECODE_STATIC_SCRATCH_BYTES];

namespace {
void *g_static_scratch[kMaxDevices] = {};
std::mutex g_static_mu;

// Device address of the static scratch on the current device. In host code the array's name only stands for the
// device symbol, so its device address is looked up once per device, with that device current, and kept. The kept
// address belongs to the device's primary context as it was at that first call (the one torch and the runtime
// use); a cudaDeviceReset afterwards would leave it stale.
int static_scratch_ptr(void **out) {
    int d = 0;
    OUMU_CK(cudaGetDevice(&d));
    if (d < 0 || d >= kMaxDevices) return OUMU_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (!g_static_scratch[d]) {
        void *p = nullptr;
        OUMU_CK(cudaGetSymbolAddress(&p, oumu_decode_static_scratch));
        g_static_scratch[d] = p;
    }
    *out = g_static_scratch[d];
    return OUMU_OK;
}
}  // namespace

extern "C" {

int oumu_attn_decode_static(const void *qkv, const void *kc, const void *vc, void *out, const int *pos,
                            const int *lens, int B, int nq, int nk, int hd, int maxlen, float scale,
                            oumu_stream_t stream) {
    // every check of oumu_attn_decode first: a rejected call queues nothing on the stream and leaves the shared
    // array as it was
    int rc = decode_check(qkv, kc, vc, out, nullptr, nullptr, pos, lens, B, nq, nk, hd, maxlen, scale);
    if (rc) return rc;
    // the scratch this shape needs: the combine counters, then one partial pair per CTA (at least one CTA)
    const size_t cbytes = decode_counter_bytes(B, nk), need = cbytes + decode_part_bytes(hd);
    if (need > OUMU_DECODE_STATIC_SCRATCH_BYTES) {
        std::snprintf(g_last_cuda, sizeof(g_last_cuda),
                      "oumu_attn_decode_static: B * nk = %ld needs %zu bytes of scratch, the static scratch holds %d",
                      static_cast<long>(B) * nk, need, OUMU_DECODE_STATIC_SCRATCH_BYTES);
        return OUMU_ERR_WORKSPACE;
    }
    void *ws = nullptr;
    rc = static_scratch_ptr(&ws);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    // the counters must start at zero; the array keeps whatever the previous call (or an aborted one) left
    OUMU_CK(cudaMemsetAsync(ws, 0, cbytes, st));
    return decode_launch(false, qkv, kc, vc, out, ws, OUMU_DECODE_STATIC_SCRATCH_BYTES, nullptr, nullptr, pos, lens,
                         B, nq, nk, hd, maxlen, scale, st);
}

int oumu_attn_decode_step(void *qkv, void *kc, void *vc, void *out, void *workspace, size_t workspace_bytes,
                          const float *cos_t, const float *sin_t, const int *pos, const int *lens, int B, int nq,
                          int nk, int hd, int maxlen, float scale, oumu_stream_t stream) {
    return decode_entry(true, qkv, kc, vc, out, workspace, workspace_bytes, cos_t, sin_t, pos, lens, B, nq, nk, hd,
                        maxlen, scale, stream);
}

int oumu_attn_full(const void *qkv, void *out, int rows, int seq, int causal, int nq, int nk, int hd, float scale,
                   oumu_stream_t stream) {
    if (!qkv || !out || rows < 0 || seq < 1 || nq < 1 || nk < 1 || nq % nk || !(scale > 0.f)) return OUMU_ERR_INVALID;
    if (rows % seq) return OUMU_ERR_INVALID;
    if (!head_dim_ok(hd)) return OUMU_ERR_UNSUPPORTED;
    if (!aligned16(qkv) || !aligned16(out)) return OUMU_ERR_INVALID;
    if (rows == 0) return OUMU_OK;
    int sms = 0;
    int rc = current_device(&sms);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (seq <= fs::ROWS) {
        if (small_use_tc(rows, seq, nq, nk, sms))
            return hd == 128 ? launch_small_tc<128>(qkv, out, rows, seq, causal, nq, nk, scale, sms, st)
                             : launch_small_tc<64>(qkv, out, rows, seq, causal, nq, nk, scale, sms, st);
        return hd == 128 ? launch_small<128>(qkv, out, rows, seq, causal, nq, nk, scale, sms, st)
                         : launch_small<64>(qkv, out, rows, seq, causal, nq, nk, scale, sms, st);
    }
    return hd == 128 ? launch_prefill<128>(qkv, out, rows, seq, causal, nq, nk, scale, st)
                     : launch_prefill<64>(qkv, out, rows, seq, causal, nq, nk, scale, st);
}

int oumu_attn_full_rope(const void *qkv, void *out, const float *cos_t, const float *sin_t, int rows, int seq,
                        int causal, int nq, int nk, int hd, float scale, oumu_stream_t stream) {
    if (!qkv || !out || !cos_t || !sin_t || rows < 0 || seq < 1 || nq < 1 || nk < 1 || nq % nk || !(scale > 0.f))
        return OUMU_ERR_INVALID;
    if (rows % seq) return OUMU_ERR_INVALID;
    if (!head_dim_ok(hd)) return OUMU_ERR_UNSUPPORTED;
    if (seq > fs::ROWS || nq / nk < 2 || (nq / nk) * seq > fs::MAXM) return OUMU_ERR_UNSUPPORTED;
    if (!aligned16(qkv) || !aligned16(out) || !aligned16(cos_t) || !aligned16(sin_t)) return OUMU_ERR_INVALID;
    if (rows == 0) return OUMU_OK;
    int sms = 0;
    int rc = current_device(&sms);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (small_use_tc(rows, seq, nq, nk, sms))
        return hd == 128 ? launch_small_tc<128>(qkv, out, rows, seq, causal, nq, nk, scale, sms, st, cos_t, sin_t)
                         : launch_small_tc<64>(qkv, out, rows, seq, causal, nq, nk, scale, sms, st, cos_t, sin_t);
    return hd == 128 ? launch_small<128>(qkv, out, rows, seq, causal, nq, nk, scale, sms, st, cos_t, sin_t)
                     : launch_small<64>(qkv, out, rows, seq, causal, nq, nk, scale, sms, st, cos_t, sin_t);
}

int oumu_attn_prefill_kv(const void *qkv, void *out, void *kc, void *vc, int T, int slots, int nq, int nk, int hd,
                         int maxlen, float scale, oumu_stream_t stream) {
    if (!qkv || !out || !kc || !vc || T < 1 || slots < 1 || nq < 1 || nk < 1 || nq % nk || maxlen < T ||
        !(scale > 0.f))
        return OUMU_ERR_INVALID;
    if (!head_dim_ok(hd)) return OUMU_ERR_UNSUPPORTED;
    if (T <= fs::ROWS) return OUMU_ERR_UNSUPPORTED;  // the tensor-core path only (prompts longer than 16)
    if (!aligned16(qkv) || !aligned16(out) || !aligned16(kc) || !aligned16(vc)) return OUMU_ERR_INVALID;
    int sms = 0;
    int rc = current_device(&sms);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    return hd == 128 ? launch_prefill<128>(qkv, out, T, T, 1, nq, nk, scale, st, kc, vc, slots, maxlen)
                     : launch_prefill<64>(qkv, out, T, T, 1, nq, nk, scale, st, kc, vc, slots, maxlen);
}

int oumu_kv_replicate(void *cache, int B, int nk, int maxlen, int hd, int T, oumu_stream_t stream) {
    if (!cache || B < 1 || nk < 1 || maxlen < 1 || T < 0 || T > maxlen) return OUMU_ERR_INVALID;
    if (!head_dim_ok(hd)) return OUMU_ERR_UNSUPPORTED;
    if (!aligned16(cache)) return OUMU_ERR_INVALID;
    if (B == 1 || T == 0) return OUMU_OK;
    const int spg = 8;
    const long total = static_cast<long>(T) * nk * (hd / 8);
    dim3 grid(static_cast<unsigned>((total + 255) / 256), static_cast<unsigned>((B - 1 + spg - 1) / spg));
    k_kv_replicate<<<grid, 256, 0, stream>>>(static_cast<bf16 *>(cache), B, nk, maxlen, hd, T, spg);
    OUMU_CK(cudaGetLastError());
    return OUMU_OK;
}

int oumu_set_wait_limit_ns(unsigned long long ns) {
    const unsigned long long v = ns ? ns : OUMU_WAIT_LIMIT_DEFAULT_NS;
    OUMU_CK(cudaMemcpyToSymbol(oumu_wait_limit_ns, &v, sizeof(v)));
    return OUMU_OK;
}

int oumu_test_drop_last_tile(int on) { return g_drop_tile.exchange(on ? 1 : 0); }

int oumu_device_error(int reset) {
    unsigned int v = 0;
    OUMU_CK(cudaMemcpyFromSymbol(&v, oumu_dev_error, sizeof(v)));
    if (reset) {
        unsigned int z = 0;
        OUMU_CK(cudaMemcpyToSymbol(oumu_dev_error, &z, sizeof(z)));
    }
    return static_cast<int>(v);
}

// ------------------------------------------------------------------------------------------------------------
// Step glue (include/oumu_step.h)
// ------------------------------------------------------------------------------------------------------------

int oumu_rmsnorm(void *res, const void *d, const void *w, void *out, int rows, int dim, float eps,
                 oumu_stream_t stream) {
    if (!res || !w || !out || rows < 0) return OUMU_ERR_INVALID;
    if (dim != 1024 && dim != 2048) return OUMU_ERR_UNSUPPORTED;
    if (!aligned16(res) || !aligned16(w) || !aligned16(out) || (d && !aligned16(d))) return OUMU_ERR_INVALID;
    if (rows == 0) return OUMU_OK;
    const unsigned grid = static_cast<unsigned>(rows);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (dim == 1024)
        OUMU_CK(launch_k(glue::k_rmsnorm<1024>, dim3(grid), dim3(128), 0, st, static_cast<bf16 *>(res),
                         static_cast<const bf16 *>(d), static_cast<const bf16 *>(w), static_cast<bf16 *>(out), rows,
                         eps));
    else
        OUMU_CK(launch_k(glue::k_rmsnorm<2048>, dim3(grid), dim3(256), 0, st, static_cast<bf16 *>(res),
                         static_cast<const bf16 *>(d), static_cast<const bf16 *>(w), static_cast<bf16 *>(out), rows,
                         eps));
    return OUMU_OK;
}

int oumu_silu_mul(const void *gu, void *out, int rows, int F, oumu_stream_t stream) {
    if (!gu || !out || rows < 0 || F < 8 || F % 8) return OUMU_ERR_INVALID;
    if (!aligned16(gu) || !aligned16(out)) return OUMU_ERR_INVALID;
    const long vecs = static_cast<long>(rows) * (F / 8);
    if (vecs == 0) return OUMU_OK;
    OUMU_CK(launch_k(glue::k_silu_mul, dim3(static_cast<unsigned>((vecs + 255) / 256)), dim3(256), 0,
                     reinterpret_cast<cudaStream_t>(stream), static_cast<const bf16 *>(gu), static_cast<bf16 *>(out),
                     rows, F));
    return OUMU_OK;
}

int oumu_pointwise(void *x, long n, int op, float scale, oumu_stream_t stream) {
    if (!x || n < 0 || n % 8 || (op != 0 && op != 1) || !aligned16(x)) return OUMU_ERR_INVALID;
    if (op == 1 && !(scale != 0.f)) return OUMU_ERR_INVALID;
    if (n == 0) return OUMU_OK;
    const long vecs = n / 8;
    OUMU_CK(launch_k(glue::k_pointwise, dim3(static_cast<unsigned>((vecs + 255) / 256)), dim3(256), 0,
                     reinterpret_cast<cudaStream_t>(stream), static_cast<bf16 *>(x), n, op, scale));
    return OUMU_OK;
}

int oumu_build_seq(void *seq_out, const void *mu, const void *temb, const void *condp, const void *xp, int rows,
                   int B, int seq, int H, oumu_stream_t stream) {
    if (!seq_out || !temb || !xp || rows < 0 || H < 8 || H % 8) return OUMU_ERR_INVALID;
    if (seq == 11) {
        if (!mu || !condp || B < 0 || rows != 2 * B || !aligned16(mu) || !aligned16(condp)) return OUMU_ERR_INVALID;
    } else if (seq != 5) {
        return OUMU_ERR_UNSUPPORTED;
    }
    if (!aligned16(seq_out) || !aligned16(temb) || !aligned16(xp)) return OUMU_ERR_INVALID;
    const long vecs = static_cast<long>(rows) * seq * (H / 8);
    if (vecs == 0) return OUMU_OK;
    glue::k_build_seq<<<static_cast<unsigned>((vecs + 255) / 256), 256, 0, stream>>>(
        static_cast<bf16 *>(seq_out), static_cast<const bf16 *>(mu), static_cast<const bf16 *>(temb),
        static_cast<const bf16 *>(condp), static_cast<const bf16 *>(xp), rows, B, seq, H);
    OUMU_CK(cudaGetLastError());
    return OUMU_OK;
}

int oumu_cfg_euler(void *x, const void *out, int B, int seq, int first, float dt, float cfg, oumu_stream_t stream) {
    if (!x || !out || B < 0 || seq < 4 || first < 0 || first + 4 > seq) return OUMU_ERR_INVALID;
    if (B == 0) return OUMU_OK;
    glue::k_cfg_euler<<<static_cast<unsigned>(B), 256, 0, stream>>>(static_cast<bf16 *>(x),
                                                                    static_cast<const bf16 *>(out), B, seq, first,
                                                                    dt, cfg);
    OUMU_CK(cudaGetLastError());
    return OUMU_OK;
}

int oumu_step_end(const void *stop_logits, const void *patch, void *patches, int *stop, int *ctr, int *lens, int B,
                  int min_len, int max_steps, oumu_stream_t stream) {
    if (!stop_logits || !patch || !patches || !stop || !ctr || B < 0 || max_steps < 1) return OUMU_ERR_INVALID;
    if (!aligned16(patch) || !aligned16(patches)) return OUMU_ERR_INVALID;
    glue::k_step_end<<<1, 256, 0, stream>>>(static_cast<const bf16 *>(stop_logits), static_cast<const bf16 *>(patch),
                                            static_cast<bf16 *>(patches), stop, ctr, lens, B, min_len, max_steps);
    OUMU_CK(cudaGetLastError());
    return OUMU_OK;
}

struct oumu_decode_loop_s {
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
};

namespace {

int add_loop_test(cudaGraphNode_t *node, cudaGraph_t g, const cudaGraphNode_t *dep, cudaGraphConditionalHandle h,
                  const int *stop, const int *ctr, int *status, int B, int max_steps, int first) {
    void *args[] = {&h, &stop, &ctr, &status, &B, &max_steps, &first};
    cudaKernelNodeParams kp = {};  // shared memory 0, no extra launch options
    kp.func = reinterpret_cast<void *>(glue::k_loop_test);
    kp.gridDim = dim3(1);
    kp.blockDim = dim3(256);
    kp.kernelParams = args;
    OUMU_CK(cudaGraphAddKernelNode(node, g, dep, dep ? 1 : 0, &kp));
    return OUMU_OK;
}

int build_loop(oumu_decode_loop_s *L, cudaGraph_t step, const int *stop, const int *ctr, int *status, int B,
               int max_steps) {
    OUMU_CK(cudaGraphCreate(&L->graph, 0));
    cudaGraphConditionalHandle h;
    OUMU_CK(cudaGraphConditionalHandleCreate(&h, L->graph, 0, 0));
    cudaGraphNode_t pre, loop, child, test;
    int rc = add_loop_test(&pre, L->graph, nullptr, h, stop, ctr, status, B, max_steps, 1);
    if (rc) return rc;
    alignas(cudaGraphNodeParams) unsigned char raw[sizeof(cudaGraphNodeParams)] = {};  // zeroed: reserved fields
    auto *cp = reinterpret_cast<cudaGraphNodeParams *>(raw);
    cp->type = cudaGraphNodeTypeConditional;
    cp->conditional.handle = h;
    cp->conditional.type = cudaGraphCondTypeWhile;
    cp->conditional.size = 1;
    OUMU_CK(cudaGraphAddNode(&loop, L->graph, &pre, 1, cp));
    cudaGraph_t body = cp->conditional.phGraph_out[0];
    OUMU_CK(cudaGraphAddChildGraphNode(&child, body, nullptr, 0, step));
    rc = add_loop_test(&test, body, &child, h, stop, ctr, status, B, max_steps, 0);
    if (rc) return rc;
    OUMU_CK(cudaGraphInstantiate(&L->exec, L->graph, 0));
    return OUMU_OK;
}

}  // namespace

int oumu_decode_loop_create(void *step_graph, const int *stop, const int *ctr, int *status, int B, int max_steps,
                            oumu_decode_loop_t *loop) {
    if (!loop) return OUMU_ERR_INVALID;
    *loop = nullptr;
    if (!step_graph || !stop || !ctr || !status || B < 1 || max_steps < 1) return OUMU_ERR_INVALID;
    auto *L = new oumu_decode_loop_s;
    const int rc = build_loop(L, static_cast<cudaGraph_t>(step_graph), stop, ctr, status, B, max_steps);
    if (rc) {
        oumu_decode_loop_destroy(L);
        return rc;
    }
    *loop = L;
    return OUMU_OK;
}

int oumu_decode_loop_launch(oumu_decode_loop_t loop, oumu_stream_t stream) {
    if (!loop || !loop->exec) return OUMU_ERR_INVALID;
    OUMU_CK(cudaGraphLaunch(loop->exec, reinterpret_cast<cudaStream_t>(stream)));
    return OUMU_OK;
}

int oumu_decode_loop_destroy(oumu_decode_loop_t loop) {
    if (!loop) return OUMU_OK;
    cudaError_t e1 = cudaSuccess, e2 = cudaSuccess;
    if (loop->exec) e1 = cudaGraphExecDestroy(loop->exec);
    if (loop->graph) e2 = cudaGraphDestroy(loop->graph);
    delete loop;
    OUMU_CK(e1);
    OUMU_CK(e2);
    return OUMU_OK;
}

int oumu_gemm(const void *x, int ldx, const void *w, void *y, int ldy, const void *bias, int M, int N, int K,
              oumu_stream_t stream) {
    if (!gemm_args_ok(x, ldx, w, y, ldy, M, N, K)) return OUMU_ERR_INVALID;
    int sms = 0, dev = 0;
    int rc = current_device(&sms);
    if (rc) return rc;
    OUMU_CK(cudaGetDevice(&dev));
    const GemmShape gs = gemm_shape(M, N, K);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (gs.tn == 32) return launch_gemm<32, kGemmStages32>(x, ldx, w, y, ldy, bias, M, N, K, gs, dev, st);
    if (gs.tn == 64) return launch_gemm<64, kGemmStages64>(x, ldx, w, y, ldy, bias, M, N, K, gs, dev, st);
    return launch_gemm<128, kGemmStages128>(x, ldx, w, y, ldy, bias, M, N, K, gs, dev, st);
}

int oumu_gemm_swiglu(const void *x, int ldx, const void *w_il, void *act, int ldact, const void *bias_il, int M,
                     int F, int K, oumu_stream_t stream) {
    if (F < 8 || F % 8 != 0 || F > (1 << 29)) return OUMU_ERR_INVALID;
    const int N = 2 * F;
    // the act rows are F wide: the checks of the plain form with its N, then the output's own pitch
    if (!gemm_args_ok(x, ldx, w_il, act, N, M, N, K) || ldact < F) return OUMU_ERR_INVALID;
    int sms = 0, dev = 0;
    int rc = current_device(&sms);
    if (rc) return rc;
    OUMU_CK(cudaGetDevice(&dev));
    const GemmShape gs = gemm_shape(M, N, K);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (gs.tn == 32) return launch_gemm<32, kGemmStages32>(x, ldx, w_il, act, ldact, bias_il, M, N, K, gs, dev, st, 1);
    if (gs.tn == 64) return launch_gemm<64, kGemmStages64>(x, ldx, w_il, act, ldact, bias_il, M, N, K, gs, dev, st, 1);
    return launch_gemm<128, kGemmStages128>(x, ldx, w_il, act, ldact, bias_il, M, N, K, gs, dev, st, 1);
}

}  // extern "C"
