// vtx_fa.cu — C ABI entry points (include/vtx_fa.h): operand validation,
// kernel selection, TMA descriptor encoding and workspace accounting.
//
// Path selection for vtx_flash_attn_ext (the ggml_flash_attn_ext node of
// src/voxtral.cpp:1611 / :1802):
//   * many query rows (n_q * Hq/Hkv >= 64) and head_dim 64/128
//       -> fa_prefill_sm100_kernel (tcgen05 + TMEM + TMA).  F16 K/V whose
//          strides TMA can address are read in place; F32 / Q8_0 / oddly
//          strided K/V are first converted to a packed f16 copy in the
//          workspace (what ggml-cuda does for non-F16 caches too).
//   * otherwise (decode, short chunks) -> fa_splitkv_kernel on the native
//     K/V dtype + fa_combine_kernel when the keys are split.
// Nothing here allocates, synchronises or aborts.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <atomic>
#include <mutex>
#include <utility>
#include <vector>

#include "../../include/vtx_fa.h"
#include "vtx_ptx.cuh"
#include "fa_splitkv.cuh"
#include "fa_prefill_sm100.cuh"
#include "fa_encoder_sk.cuh"
#include "fa_decode_mma.cuh"
#include "fa_decode_q8.cuh"
#include "fa_decode_f32.cuh"
#include "kv_append.cuh"
#include "enc_stitch.cuh"
#include "out_proj.cuh"
#include "decode_layer.cuh"

using namespace vtx;

// Device-side error word written by bounded waits that ran out (see
// vtx_ptx.cuh).  One per device, read and cleared by vtx_read_device_error.
__device__ int g_vtx_kernel_err;

namespace {

constexpr int kMaxDevices = 64;

struct DeviceState {
    int ok = 0;
    int sms = 148;
    int *err = nullptr;
};
DeviceState g_dev[kMaxDevices];
std::once_flag g_dev_once[kMaxDevices];
std::once_flag g_encode_once;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

// Per-device set-up runs exactly once (std::call_once), so concurrent first
// calls from several host threads are ordered: every caller sees the state
// the one initialising call wrote.
int ensure_device(DeviceState **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return VTX_ERR_NO_DEVICE;
    DeviceState &s = g_dev[dev];
    std::call_once(g_dev_once[dev], [&] {
        int major = 0, minor = 0;
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
        cudaDeviceGetAttribute(&s.sms, cudaDevAttrMultiProcessorCount, dev);
        s.ok = (major == 10 && minor == 0);
        void *p = nullptr;
        if (s.ok && cudaGetSymbolAddress(&p, g_vtx_kernel_err) != cudaSuccess) s.ok = 0;
        s.err = static_cast<int *>(p);
        if (s.ok) {
            std::call_once(g_encode_once, [] {
                cudaDriverEntryPointQueryResult q;
                void *fn = nullptr;
                if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
                    q == cudaDriverEntryPointSuccess)
                    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
            });
        }
        cudaGetLastError();
    });
    if (!s.ok) return VTX_ERR_NO_DEVICE;
    *out = &s;
    return VTX_OK;
}

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
inline int elem_size(int t) { return t == VTX_TYPE_F32 ? 4 : 2; }
inline int row_bytes(int t, int64_t d) { return t == VTX_TYPE_Q8_0 ? (int)(d / 32 * 34) : (int)(d * elem_size(t)); }

// ---- operand checks ----------------------------------------------------------

struct Geo {
    int D, n_q, n_kv, Hq, Hkv, G, B, Bkv;
    int kv_type;
};

int check_operands(const vtx_tensor *q, const vtx_tensor *k, const vtx_tensor *v, const vtx_tensor *mask,
                   const vtx_fa_params *p, const vtx_tensor *dst, Geo *g) {
    if (!q || !k || !v || !p) return VTX_ERR_NULL;
    if (q->type != VTX_TYPE_F32 && q->type != VTX_TYPE_F16) return VTX_ERR_TYPE;
    if (k->type != v->type) return VTX_ERR_TYPE;
    if (k->type != VTX_TYPE_F32 && k->type != VTX_TYPE_F16 && k->type != VTX_TYPE_Q8_0) return VTX_ERR_TYPE;
    for (int i = 0; i < 4; ++i)
        if (q->ne[i] < 0 || k->ne[i] < 0 || v->ne[i] < 0) return VTX_ERR_SHAPE;
    if (q->ne[0] != k->ne[0] || v->ne[0] != k->ne[0]) return VTX_ERR_SHAPE;
    if (k->ne[1] != v->ne[1] || k->ne[2] != v->ne[2] || k->ne[3] != v->ne[3]) return VTX_ERR_SHAPE;
    if (k->ne[2] == 0 || q->ne[2] % k->ne[2] != 0) return VTX_ERR_SHAPE;
    if (k->ne[3] == 0 || q->ne[3] % k->ne[3] != 0) return VTX_ERR_SHAPE;
    const int64_t D = q->ne[0];
    if (D != 64 && D != 128) return VTX_ERR_UNSUPPORTED;
    if (q->ne[1] > INT32_MAX || k->ne[1] > INT32_MAX || q->ne[2] > 65535 || q->ne[3] > 65535) return VTX_ERR_SHAPE;
    if ((size_t)q->nb[0] != (size_t)elem_size(q->type)) return VTX_ERR_STRIDE;
    if (k->type == VTX_TYPE_Q8_0) {
        if (k->nb[0] != 34 || v->nb[0] != 34) return VTX_ERR_STRIDE;
    } else if (k->nb[0] != (size_t)elem_size(k->type) || v->nb[0] != (size_t)elem_size(v->type)) {
        return VTX_ERR_STRIDE;
    }
    if (p->window < 0 || (p->window > 0 && !p->causal)) return VTX_ERR_UNSUPPORTED;
    if (!std::isfinite(p->scale) || !std::isfinite(p->max_bias) || !std::isfinite(p->logit_softcap))
        return VTX_ERR_UNSUPPORTED;
    if (dst) {
        // F32 is ggml's result type; F16 (the tcgen05 prefill/encoder path only)
        // is the same result rounded as ggml rounds the activations of the F16
        // output-projection weight that consumes it
        if (dst->type != VTX_TYPE_F32 && dst->type != VTX_TYPE_F16) return VTX_ERR_TYPE;
        if (dst->ne[0] != v->ne[0] || dst->ne[1] != q->ne[2] || dst->ne[2] != q->ne[1] || dst->ne[3] != q->ne[3])
            return VTX_ERR_SHAPE;
        if (dst->nb[0] != (size_t)elem_size(dst->type) || dst->nb[1] % 16 || dst->nb[2] % 16 || dst->nb[3] % 16)
            return VTX_ERR_STRIDE;
    }
    if (mask) {
        if (mask->type != VTX_TYPE_F16) return VTX_ERR_TYPE;
        if (mask->ne[0] < k->ne[1] || mask->ne[1] < q->ne[1]) return VTX_ERR_SHAPE;
        if (mask->ne[2] <= 0 || mask->ne[3] <= 0 || q->ne[2] % mask->ne[2] || q->ne[3] % mask->ne[3])
            return VTX_ERR_SHAPE;
        if (mask->nb[0] != 2) return VTX_ERR_STRIDE;
    }
    g->D = (int)D;
    g->n_q = (int)q->ne[1];
    g->n_kv = (int)k->ne[1];
    g->Hq = (int)q->ne[2];
    g->Hkv = (int)k->ne[2];
    g->G = g->Hq / g->Hkv;
    g->B = (int)q->ne[3];
    g->Bkv = (int)k->ne[3];
    g->kv_type = k->type;
    return VTX_OK;
}

// ---- plans ---------------------------------------------------------------------

struct SplitPlan {
    int maxr, tok_per_cta, hc, n_hchunks, n_qtiles, chunk, n_splits, tk;
    size_t part_bytes;     // partial (o, m, l) workspace
};

int largest_divisor_le(int n, int cap) {
    for (int d = cap; d >= 1; --d)
        if (n % d == 0) return d;
    return 1;
}

// streaming: the work goes to the warp-per-item decode kernels (F16 / Q8_0),
// whose splits need only be multiples of their 16-key stage.  Batched decode
// is planned for max_kv (the caller's bound), not the lengths it will see, so
// with few streams short caches would leave most of the GPU idle: streaming
// plans aim at ~16 work items per SM at any length (32-key splits for one
// stream over an 8192-row window), large batches keep their 1024-key chunks.
// streaming: the F16 decode kernel (a warp per head and split) runs.
// q8_ctas: the Q8_0 decode kernel runs with this many CTAs per key split
// (streams x head groups); each CTA holds an SM, so the keys are split for
// about one CTA per SM, in 16-key stages, at least two stages per CTA.
SplitPlan plan_split(const Geo &g, int sms, int max_kv, bool batched, bool streaming = false, int q8_ctas = 0) {
    SplitPlan s{};
    s.tk = (streaming || q8_ctas) ? 16 : g.kv_type == VTX_TYPE_F32 ? 32 : 64;
    s.maxr = (g.n_q * g.G <= 4 && g.G <= 4) ? 4 : 16;
    s.hc = largest_divisor_le(g.G, s.maxr);
    s.n_hchunks = g.G / s.hc;
    s.tok_per_cta = std::max(1, s.maxr / s.hc);
    s.n_qtiles = (g.n_q + s.tok_per_cta - 1) / s.tok_per_cta;
    const long long base = (long long)g.B * g.Hkv * s.n_hchunks * s.n_qtiles;
    const int kv = std::max(1, max_kv);
    const int max_tiles = (kv + s.tk - 1) / s.tk;
    long long want = (4LL * sms + base - 1) / base;     // ~4 CTAs per SM in flight
    if (batched) want = std::max<long long>(want, (kv + 1023) / 1024);
    if (streaming) want = std::max<long long>(want, (16LL * sms + base - 1) / base);
    if (q8_ctas) want = std::max<long long>((sms + q8_ctas - 1) / q8_ctas, batched ? (kv + 1023) / 1024 : 1);
    int n_splits = (int)std::min<long long>(std::max<long long>(want, 1), max_tiles);
    int chunk_tiles = (max_tiles + n_splits - 1) / n_splits;
    if (q8_ctas) chunk_tiles = std::max(chunk_tiles, 2);
    s.chunk = chunk_tiles * s.tk;
    s.n_splits = (kv + s.chunk - 1) / s.chunk;
    s.part_bytes = 0;
    if (s.n_splits > 1) {
        const size_t work = (size_t)base * s.n_splits * s.maxr;
        s.part_bytes = align_up(work * g.D * 4, 256) + align_up(work * 2 * 4, 256);
    }
    return s;
}

struct PrefillPlan {
    bool use = false;
    bool convert = false;      // K/V copied to packed f16 in the workspace
    int nqt = 1, tok_per_tile = 0, n_tiles_q = 0, n_cta_q = 0;
    size_t conv_bytes = 0;
};

bool tma_ok(const vtx_tensor *t) {
    const uintptr_t base = reinterpret_cast<uintptr_t>(t->data);
    if (base % 16) return false;
    for (int i = 1; i < 4; ++i)
        if (t->ne[i] > 1 && (t->nb[i] % 16 || t->nb[i] >= (1ULL << 40))) return false;
    return true;
}

bool q_rows_aligned(const vtx_tensor *q) {
    const uintptr_t base = reinterpret_cast<uintptr_t>(q->data);
    if (base % 16) return false;
    for (int i = 1; i < 4; ++i)
        if (q->ne[i] > 1 && q->nb[i] % 16) return false;
    return true;
}

PrefillPlan plan_prefill(const Geo &g, const vtx_tensor *q, const vtx_tensor *k, const vtx_tensor *v, int sms,
                         bool causal) {
    PrefillPlan p;
    if (g.G > 128) return p;
    if ((long long)g.n_q * g.G < 64) return p;
    if (!q_rows_aligned(q)) return p;
    p.use = true;
    p.convert = !(g.kv_type == VTX_TYPE_F16 && tma_ok(k) && tma_ok(v));
    p.tok_per_tile = 128 / g.G;
    p.n_tiles_q = (g.n_q + p.tok_per_tile - 1) / p.tok_per_tile;
    const long long ctas2 = (long long)((p.n_tiles_q + 1) / 2) * g.Hkv * g.B;
    // Two Q tiles per CTA share every K/V tile and ping-pong the tensor core
    // (one tile's softmax overlaps the other's MMAs); a single tile per CTA
    // serialises MMA and softmax and is kept for grids too small to fill the
    // SMs with pairs.  (Measured with the longest-first order of causal grids:
    // window-750 encoder chunk 29.6 us with pairs vs 39.0 us with single tiles,
    // 8192-token causal prefill 543 vs 715 us.)
    (void)causal;
    p.nqt = (p.n_tiles_q >= 2 && ctas2 >= (sms * 3) / 4) ? 2 : 1;
    p.n_cta_q = (p.n_tiles_q + p.nqt - 1) / p.nqt;
    if (p.convert) p.conv_bytes = 2 * align_up((size_t)g.Bkv * g.Hkv * g.n_kv * g.D * 2, 256);
    return p;
}

// Persistent encoder kernel (fa_encoder_sk.cuh): the bidirectional head_dim
// 64 node with f16 Q / K / V read in place and no mask tensor, softcap or
// causal flag -- the offline encoder (src/voxtral.cpp:1611) -- when its
// per-pair grid would take more than one wave (several clips per call).  One
// CTA per SM, each taking an equal share of the (Q-tile pair, key tile) work.  Workspace: a merge flag per
// (CTA, Q tile), the producers' row maxima and sums, their partial O rows.
struct SkPlan {
    bool use = false;
    int ctas = 0, n_pairs = 0, n_iter = 0;
    int total = 0;
    int bound[kSkMaxCtas + 1];
    size_t flags_bytes = 0, part_bytes = 0;
    size_t bytes() const { return use ? flags_bytes + part_bytes : 0; }
};

SkPlan plan_sk(const Geo &g, const PrefillPlan &pp, int q_type, int causal, float scale, float softcap, int sms) {
    SkPlan p;
    if (!pp.use || pp.convert || g.D != 64 || q_type != VTX_TYPE_F16 || g.kv_type != VTX_TYPE_F16) return p;
    if (causal || softcap != 0.0f || !(scale > 0.0f) || pp.n_tiles_q < 2 || g.n_kv <= 0 || 128 % g.G) return p;
    p.n_pairs = (pp.n_tiles_q + 1) / 2;
    // One wave of per-pair CTAs (one clip of the offline encoder: 120 CTAs)
    // runs faster on the per-pair kernel: a split pair's merge costs its
    // owner ~2-4 us of memory round trips, about what the idle SMs would save
    // (measured, 1500 x 1500 x 20 heads: 29.0 vs 23.9 us).  Beyond one wave
    // the per-pair grid leaves a partial last wave, which this kernel avoids.
    if ((long long)g.B * g.Hkv * p.n_pairs <= sms) return p;
    p.n_iter = (g.n_kv + 127) / 128;
    const long long total = (long long)g.B * g.Hkv * p.n_pairs * p.n_iter;
    const long long ctas = std::min<long long>(std::min(sms, kSkMaxCtas), total / 4);
    if (ctas < 1 || total > 0x7fffffffLL) return p;
    p.total = (int)total;
    p.ctas = (int)ctas;
    p.flags_bytes = align_up((size_t)2 * p.ctas * sizeof(unsigned long long), 256);
    p.part_bytes = align_up((size_t)2 * p.ctas * SkCfg<64>::PGROUPS * 128 * 4 * sizeof(float), 256);
    p.use = true;
    return p;
}

// Equal contiguous ranges, one per CTA.
SkPlan plan_sk_ranges(const Geo &g, const PrefillPlan &pp, int q_type, int causal, float scale, float softcap,
                      int sms) {
    SkPlan p = plan_sk(g, pp, q_type, causal, scale, softcap, sms);
    if (p.use)
        for (int c = 0; c <= p.ctas; ++c) p.bound[c] = (int)((long long)c * p.total / p.ctas);
    return p;
}

// Map of the persistent kernel's partials: F32 [groups][128 rows][4 floats]
// (group = one column group of D/4 + 1 of one (CTA, Q tile)); one box of
// 4 x 128 x (D/4 + 1) is a (CTA, Q tile)'s whole block.
int encode_part_map(CUtensorMap *m, void *ptr, int blocks) {
    if (!g_encode) return VTX_ERR_CUDA;
    constexpr int PG = SkCfg<64>::PGROUPS;
    cuuint64_t dims[3] = {4, 128, (cuuint64_t)blocks * PG};
    cuuint64_t strides[2] = {16, 128 * 16};
    cuuint32_t box[3] = {4, 128, PG};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, ptr, dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? VTX_OK : VTX_ERR_WORKSPACE;
}

// ---- realtime encoder chunk geometry (host) -------------------------------------
// Chunk constants of src/voxtral.cpp:26-27 and the downsample factor of
// include/voxtral.h:51.
constexpr int kEncChunkMel = 3000, kEncChunkOverlap = 750, kEncDownsample = 4;

// Output length of one causal convolution (compute_causal_conv1d_dims,
// src/voxtral.cpp:1280-1297); the frame count is float arithmetic there too.
int causal_conv_out_len(int in_len, int kernel, int stride) {
    if (in_len <= 0 || kernel <= 0 || stride <= 0) return 0;
    const int pad = kernel - stride;
    const float frames = (float)(in_len - kernel + pad) / (float)stride + 1.0f;
    const int target = ((int)std::ceil(frames) - 1) * stride + (kernel - pad);
    const int padded = in_len + pad + std::max(0, target - in_len);
    return (padded - kernel) / stride + 1;
}

// Encoder tokens of a chunk of n mel frames (mel_frames_to_enc_tokens, :1300-1305).
int enc_tokens_of(int mel) {
    const int n = causal_conv_out_len(causal_conv_out_len(mel, 3, 1), 3, 2);
    return n - n % kEncDownsample;
}

// Stitched token count (compute_total_enc_tokens, :1308-1325).
int enc_tokens_total(int total_mel) {
    const int stride_mel = kEncChunkMel - 2 * kEncChunkOverlap;
    int total = 0;
    for (int off = 0, first = 1; off < total_mel; off += stride_mel, first = 0) {
        const int add = enc_tokens_of(std::min(kEncChunkMel, total_mel - off)) - (first ? 0 : kEncChunkOverlap);
        if (add <= 0) break;
        total += add;
    }
    return total;
}

// ---- conversion kernel: K/V (F32 | F16 strided | Q8_0) -> packed f16 ---------

// positions += 1, slots = (slots + 1) % window, kv_len = min(kv_len + 1, window)
__global__ void decode_advance_kernel(int32_t *pos, int32_t *slots, int32_t *kv_len, int n, int window) {
    grid_dep_wait();
    grid_dep_launch();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    if (pos) pos[i] += 1;
    if (slots) slots[i] = (slots[i] + 1) % window;
    if (kv_len) kv_len[i] = min(kv_len[i] + 1, window);
}

__global__ void convert_kv_f16_kernel(const char *src, long long nb1, long long nb2, long long nb3, int type,
                                      int D, int n_kv, int H, int Bk, __half *dst) {
    grid_dep_wait();
    grid_dep_launch();
    const long long total = (long long)Bk * H * n_kv * D;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int d = (int)(i % D);
        long long r = i / D;
        const int t = (int)(r % n_kv); r /= n_kv;
        const int h = (int)(r % H);
        const int b = (int)(r / H);
        const char *row = src + (long long)t * nb1 + (long long)h * nb2 + (long long)b * nb3;
        float x;
        if (type == VTX_TYPE_F32) x = reinterpret_cast<const float *>(row)[d];
        else if (type == VTX_TYPE_F16) x = __half2float(reinterpret_cast<const __half *>(row)[d]);
        else {
            const char *blk = row + (d / 32) * 34;
            x = __half2float(*reinterpret_cast<const __half *>(blk)) * (float)(int8_t)blk[2 + d % 32];
        }
        dst[i] = __float2half_rn(x);
    }
}

// Every kernel is launched with programmatic stream serialisation (PDL): it
// may be scheduled while the previous kernel on the stream drains, and waits
// for it in-kernel (grid_dep_wait) before touching global memory.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...) == cudaSuccess ? VTX_OK : VTX_ERR_CUDA;
}

// The same with the grid in clusters of `cs` CTAs along x.
template <typename... KArgs, typename... Args>
int launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, int cs,
                       Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)cs;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...) == cudaSuccess ? VTX_OK : VTX_ERR_CUDA;
}

int encode_kv_map(CUtensorMap *m, const void *ptr, int D, int n_kv, int H, int Bk, size_t nb1, size_t nb2,
                  size_t nb3) {
    if (!g_encode) return VTX_ERR_CUDA;
    cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)n_kv, (cuuint64_t)H, (cuuint64_t)Bk};
    cuuint64_t strides[3] = {(cuuint64_t)nb1, (cuuint64_t)(H > 1 ? nb2 : nb1 * (size_t)n_kv),
                             (cuuint64_t)(Bk > 1 ? nb3 : (H > 1 ? nb2 : nb1 * (size_t)n_kv) * (size_t)H)};
    for (int i = 0; i < 3; ++i)
        if (strides[i] % 16 || strides[i] == 0) return VTX_ERR_STRIDE;
    cuuint32_t box[4] = {64, 128, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void *>(ptr), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? VTX_OK : VTX_ERR_STRIDE;
}

// Q map for the prefill's TMA loads: f16 [D, Hq, n_q, B] (ggml's q strides
// nb2 = head, nb1 = token, nb3 = batch) with boxes of 64 columns x G heads x
// tok_per_tile tokens: one 128-row Q tile, rows token * G + head, in the
// 128-byte swizzle of the K tiles.  VTX_ERR_STRIDE when Q cannot be described
// (the softmax warps then copy Q themselves).
int encode_q_map(CUtensorMap *m, const void *ptr, int D, int Hq, int n_q, int B, size_t nb1, size_t nb2, size_t nb3,
                 int G, int tok_per_tile) {
    if (!g_encode) return VTX_ERR_CUDA;
    if (reinterpret_cast<uintptr_t>(ptr) % 16 || G * tok_per_tile != 128) return VTX_ERR_STRIDE;
    const size_t s1 = Hq > 1 ? nb2 : (size_t)D * 2;          // extent-1 dimensions: any legal stride
    const size_t s2 = n_q > 1 ? nb1 : s1 * (size_t)Hq;
    const size_t s3 = B > 1 ? nb3 : s2 * (size_t)n_q;
    cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)Hq, (cuuint64_t)n_q, (cuuint64_t)B};
    cuuint64_t strides[3] = {(cuuint64_t)s1, (cuuint64_t)s2, (cuuint64_t)s3};
    for (int i = 0; i < 3; ++i)
        if (strides[i] % 16 || strides[i] == 0 || strides[i] >= (1ULL << 40)) return VTX_ERR_STRIDE;
    cuuint32_t box[4] = {64, (cuuint32_t)G, (cuuint32_t)tok_per_tile, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void *>(ptr), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? VTX_OK : VTX_ERR_STRIDE;
}

// Output map for the prefill epilogue's TMA stores: F32 [D, Hq, n_q, B] with
// boxes of 32 columns x G heads x tok_per_tile tokens (one 128-row Q tile).
// Returns VTX_ERR_STRIDE when the destination cannot be described (base or
// strides not 16-byte multiples); the caller then uses plain stores.
int encode_out_map(CUtensorMap *m, void *ptr, int D, int Hq, int n_q, int B, size_t nb1, size_t nb2, size_t nb3,
                   int G, int tok_per_tile, bool f16 = false) {
    if (!g_encode) return VTX_ERR_CUDA;
    if (reinterpret_cast<uintptr_t>(ptr) % 16 || G > 256 || tok_per_tile > 256) return VTX_ERR_STRIDE;
    const size_t s1 = Hq > 1 ? nb1 : (size_t)D * (f16 ? 2 : 4);   // extent-1 dimensions: any legal stride
    const size_t s2 = n_q > 1 ? nb2 : s1 * (size_t)Hq;
    const size_t s3 = B > 1 ? nb3 : s2 * (size_t)n_q;
    cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)Hq, (cuuint64_t)n_q, (cuuint64_t)B};
    cuuint64_t strides[3] = {(cuuint64_t)s1, (cuuint64_t)s2, (cuuint64_t)s3};
    for (int i = 0; i < 3; ++i)
        if (strides[i] % 16 || strides[i] == 0) return VTX_ERR_STRIDE;
    // one box = 128 bytes of a row (32 floats or 64 halves) x the tile's rows
    cuuint32_t box[4] = {f16 ? 64u : 32u, (cuuint32_t)G, (cuuint32_t)tok_per_tile, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = g_encode(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, ptr, dims,
                          strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? VTX_OK : VTX_ERR_STRIDE;
}

void fill_math(float scale, float max_bias, float softcap, int Hq, float *qk_scale, float *softcap_out, float *m0,
               float *m1, int *n_head_log2) {
    *n_head_log2 = 1 << (int)std::floor(std::log2((double)Hq));
    *m0 = std::pow(2.0f, -(max_bias) / (float)*n_head_log2);
    *m1 = std::pow(2.0f, -(max_bias / 2.0f) / (float)*n_head_log2);
    *softcap_out = softcap;
    *qk_scale = softcap != 0.0f ? scale / softcap : scale;
}

// The combine kernel's row space: one warp per (stream, y, q tile, row of the
// tile), rows past n_q or the group included; gy = KV heads x head chunks.
// The combine kernel's row space: one CTA per (stream, y, q tile, row of the
// tile), rows past n_q or the group included; gy = KV heads x head chunks.
// Many splits (a few streams): 512 threads, so each thread merges few splits.
template <int D, int MAXR>
int launch_combine(const SplitArgs &a, int gy, cudaStream_t st) {
    const long long rows = (long long)a.B * gy * a.n_qtiles * a.tok_per_cta * a.hc;
    if (rows > 0x7fffffffLL) return VTX_ERR_UNSUPPORTED;
    const int rc = a.n_splits > 32
                       ? launch_pdl(fa_combine_kernel<D, MAXR, 512>, dim3((unsigned)rows), dim3(512), 0, st, a, gy)
                       : launch_pdl(fa_combine_kernel<D, MAXR, 128>, dim3((unsigned)rows), dim3(128), 0, st, a, gy);
    return rc == VTX_OK ? VTX_OK : VTX_ERR_CUDA;
}

template <int D, int KVT, int MAXR>
int launch_split_t(const SplitArgs &a, dim3 grid, cudaStream_t st) {
    constexpr int smem = splitkv_smem_bytes<D, KVT, MAXR>();
    static std::atomic<int> attr_done[kMaxDevices];
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_done[dev].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(fa_splitkv_kernel<D, KVT, MAXR>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess)
            return VTX_ERR_CUDA;
        attr_done[dev].store(1, std::memory_order_release);
    }
    if (launch_pdl(fa_splitkv_kernel<D, KVT, MAXR>, grid, dim3(128), smem, st, a) != VTX_OK) return VTX_ERR_CUDA;
    if (!a.write_final) {
        return launch_combine<D, MAXR>(a, (int)grid.y, st);
    }
    return VTX_OK;
}

template <int D, int KVT>
int launch_split_d(const SplitArgs &a, int maxr, dim3 grid, cudaStream_t st) {
    return maxr == 4 ? launch_split_t<D, KVT, 4>(a, grid, st) : launch_split_t<D, KVT, 16>(a, grid, st);
}

// Decode on the streaming mma.sync kernel: F16 K/V, n_q = 1, at most 4 query
// heads per KV head, 16-byte aligned rows; partials merged by the combine.
template <int D>
int launch_decode_mma_t(const SplitArgs &a, cudaStream_t st) {
    using C = DecodeCfg<D>;
    static std::atomic<int> attr_done[kMaxDevices];
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_done[dev].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(fa_decode_mma_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
            cudaSuccess)
            return VTX_ERR_CUDA;
        attr_done[dev].store(1, std::memory_order_release);
    }
    const long long items = (long long)a.B * a.Hkv * a.n_splits;
    if (launch_pdl(fa_decode_mma_kernel<D>, dim3((unsigned)((items + C::WARPS - 1) / C::WARPS)), dim3(128), C::SMEM,
                   st, a, (int)items) != VTX_OK)
        return VTX_ERR_CUDA;
    if (!a.write_final) {
        return launch_combine<D, 4>(a, a.Hkv, st);
    }
    return VTX_OK;
}

int launch_decode_mma(const SplitArgs &a, int D, cudaStream_t st) {
    return D == 64 ? launch_decode_mma_t<64>(a, st) : launch_decode_mma_t<128>(a, st);
}

// Decode over an F32 cache on the f32 streaming kernel (the reference's own
// cache type): n_q = 1, at most 4 query heads per KV head, 16-byte rows.
template <int D>
int launch_decode_f32_t(const SplitArgs &a, cudaStream_t st) {
    using C = DecodeF32Cfg<D>;
    static std::atomic<int> attr_done[kMaxDevices];
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_done[dev].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(fa_decode_f32_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
            cudaSuccess)
            return VTX_ERR_CUDA;
        attr_done[dev].store(1, std::memory_order_release);
    }
    const long long items = (long long)a.B * a.Hkv * a.n_splits;
    if ((items + C::WARPS - 1) / C::WARPS > 0x7fffffffLL) return VTX_ERR_UNSUPPORTED;
    if (launch_pdl(fa_decode_f32_kernel<D>, dim3((unsigned)((items + C::WARPS - 1) / C::WARPS)), dim3(128), C::SMEM,
                   st, a, (int)items) != VTX_OK)
        return VTX_ERR_CUDA;
    if (!a.write_final) return launch_combine<D, 4>(a, a.Hkv, st);
    return VTX_OK;
}

int launch_decode_f32(const SplitArgs &a, int D, cudaStream_t st) {
    return D == 64 ? launch_decode_f32_t<64>(a, st) : launch_decode_f32_t<128>(a, st);
}

// Q8_0 streaming decode: one CTA per (stream, group of hpc KV heads, key
// split); the heads' slices of a token row are copied as one contiguous span,
// so heads must be adjacent in the row (nb2 = one head's 136-byte row) and the
// span a multiple of 16 bytes (hpc even).  Returns hpc, or 0 when unusable.
int decode_q8_hpc(int kv_type, int D, int n_q, int G, int Hkv, int maxr, int n_hchunks, long long k_nb1,
                  long long k_nb2, long long v_nb1, long long v_nb2) {
    if (kv_type != VTX_TYPE_Q8_0 || D != 128 || n_q != 1 || G > 4 || maxr != 4 || n_hchunks != 1) return 0;
    constexpr int BLK = DecodeQ8Cfg<128>::BLK;
    if ((Hkv > 1 && (k_nb2 != BLK || v_nb2 != BLK)) || k_nb1 % 16 || v_nb1 % 16) return 0;
    for (int h = std::min(Hkv, DecodeQ8Cfg<128>::HPC_MAX); h >= 2; --h)
        if (Hkv % h == 0 && (h * BLK) % 16 == 0) return h;
    return 0;
}

int launch_decode_q8(const SplitArgs &a, int hpc, cudaStream_t st) {
    using C = DecodeQ8Cfg<128>;
    static std::atomic<int> attr_done[kMaxDevices];
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_done[dev].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(fa_decode_q8_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
            cudaSuccess)
            return VTX_ERR_CUDA;
        attr_done[dev].store(1, std::memory_order_release);
    }
    const long long items = (long long)a.B * (a.Hkv / hpc) * a.n_splits;
    if (items > 0x7fffffffLL) return VTX_ERR_UNSUPPORTED;
    if (launch_pdl(fa_decode_q8_kernel<128>, dim3((unsigned)items), dim3(C::NTHREADS), C::SMEM, st, a, hpc) != VTX_OK)
        return VTX_ERR_CUDA;
    if (!a.write_final) {
        return launch_combine<128, 4>(a, a.Hkv, st);
    }
    return VTX_OK;
}

bool decode_mma_ok(int kv_type, int n_q, int G, int vec, int maxr, int n_hchunks) {
    return kv_type == VTX_TYPE_F16 && n_q == 1 && G <= 4 && vec == 16 && maxr == 4 && n_hchunks == 1;
}

bool decode_f32_ok(int kv_type, int n_q, int G, int vec, int maxr, int n_hchunks) {
    return kv_type == VTX_TYPE_F32 && n_q == 1 && G <= 4 && vec == 16 && maxr == 4 && n_hchunks == 1;
}

int launch_split(const SplitArgs &a, int D, int kvt, int maxr, dim3 grid, cudaStream_t st) {
    if (D == 64) {
        if (kvt == VTX_TYPE_F16) return launch_split_d<64, 1>(a, maxr, grid, st);
        if (kvt == VTX_TYPE_F32) return launch_split_d<64, 0>(a, maxr, grid, st);
        return launch_split_d<64, 8>(a, maxr, grid, st);
    }
    if (kvt == VTX_TYPE_F16) return launch_split_d<128, 1>(a, maxr, grid, st);
    if (kvt == VTX_TYPE_F32) return launch_split_d<128, 0>(a, maxr, grid, st);
    return launch_split_d<128, 8>(a, maxr, grid, st);
}

int pick_vec(int row, std::initializer_list<unsigned long long> vals) {
    for (int v : {16, 8, 4}) {
        if (row % v) continue;
        bool ok = true;
        for (auto x : vals)
            if (x % (unsigned long long)v) { ok = false; break; }
        if (ok) return v;
    }
    return 0;
}

// Whether a batched decode goes to the F16 streaming kernel (the same tests
// as the dispatch below, from the batch description alone, so that the
// workspace query and the call plan the same splits).
// CTAs per key split when the Q8_0 decode kernel will run for this batch, else 0.
int batch_q8_ctas(const vtx_decode_batch *b) {
    const int G = b->n_head_q / b->n_head_kv;
    const int hpc = decode_q8_hpc(b->kv_type, b->head_dim, 1, G, b->n_head_kv, G <= 4 ? 4 : 16, 1,
                                  (long long)b->kv_nb1, (long long)b->kv_nb2, (long long)b->kv_nb1,
                                  (long long)b->kv_nb2);
    return hpc ? b->n_seq * (b->n_head_kv / hpc) : 0;
}

bool batch_streaming(const vtx_decode_batch *b) {
    const int G = b->n_head_q / b->n_head_kv;
    if (G > 4) return false;
    const int rb = row_bytes(b->kv_type, b->head_dim);
    const int vec =
        pick_vec(rb, {(unsigned long long)b->kv_nb1, (unsigned long long)(b->n_head_kv > 1 ? b->kv_nb2 : 0)});
    // F16 and F32 (warp per item); a Q8_0 CTA covers all heads of a split with
    // 211 KB of shared memory (one per SM), so its fixed cost needs the
    // coarser default splits
    return (b->kv_type == VTX_TYPE_F16 || b->kv_type == VTX_TYPE_F32) && vec == 16;
}

template <int D, int NQT, bool HM, bool UF, bool CSL = false, bool OF16 = false>
int launch_prefill_t(const CUtensorMap &mk, const CUtensorMap &mv, const CUtensorMap &mo, const CUtensorMap &mq,
                     const PrefillArgs &a, dim3 grid, cudaStream_t st) {
    using C = PrefillCfg<D, NQT>;
    static std::atomic<int> attr_done[kMaxDevices];
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_done[dev].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(fa_prefill_sm100_kernel<D, NQT, HM, UF, CSL, OF16>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
            return VTX_ERR_CUDA;
        attr_done[dev].store(1, std::memory_order_release);
    }
    return launch_pdl(fa_prefill_sm100_kernel<D, NQT, HM, UF, CSL, OF16>, grid, dim3(C::NTHREADS), C::SMEM, st, mk,
                      mv, mo, mq, a);
}

template <int D, int NQT>
int launch_prefill_d(bool hm, bool uf, const CUtensorMap &mk, const CUtensorMap &mv, const CUtensorMap &mo,
                     const CUtensorMap &mq, const PrefillArgs &a, dim3 grid, cudaStream_t st) {
    // windowed or multi-wave causal launches (flags only): the causal instantiation
    const bool csl = a.causal && !hm && !uf && (a.lpt || a.window > 0);
    if (a.o_f16) {                                            // F16 result: no mask tensor, no softcap
        if (hm || uf) return VTX_ERR_UNSUPPORTED;
        return csl ? launch_prefill_t<D, NQT, false, false, true, true>(mk, mv, mo, mq, a, grid, st)
                   : launch_prefill_t<D, NQT, false, false, false, true>(mk, mv, mo, mq, a, grid, st);
    }
    if (csl) return launch_prefill_t<D, NQT, false, false, true>(mk, mv, mo, mq, a, grid, st);
    if (uf) return hm ? launch_prefill_t<D, NQT, true, true>(mk, mv, mo, mq, a, grid, st)
                      : launch_prefill_t<D, NQT, false, true>(mk, mv, mo, mq, a, grid, st);
    return hm ? launch_prefill_t<D, NQT, true, false>(mk, mv, mo, mq, a, grid, st)
              : launch_prefill_t<D, NQT, false, false>(mk, mv, mo, mq, a, grid, st);
}

int launch_prefill(int D, int nqt, bool hm, const CUtensorMap &mk, const CUtensorMap &mv, const CUtensorMap &mo,
                   const CUtensorMap &mq, const PrefillArgs &a, dim3 grid, cudaStream_t st) {
    const bool uf = !a.fused;
    if (D == 64)
        return nqt == 2 ? launch_prefill_d<64, 2>(hm, uf, mk, mv, mo, mq, a, grid, st)
                        : launch_prefill_d<64, 1>(hm, uf, mk, mv, mo, mq, a, grid, st);
    return nqt == 2 ? launch_prefill_d<128, 2>(hm, uf, mk, mv, mo, mq, a, grid, st)
                    : launch_prefill_d<128, 1>(hm, uf, mk, mv, mo, mq, a, grid, st);
}

// The mask is not part of the workspace query, so a shape the persistent
// encoder kernel could take is sized for it; with a mask the per-pair kernel
// runs and needs less.
size_t workspace_for(const Geo &g, const vtx_tensor *q, const vtx_tensor *k, const vtx_tensor *v,
                     const vtx_fa_params *p, int sms) {
    if (g.n_q == 0) return 0;
    const PrefillPlan pp = plan_prefill(g, q, k, v, sms, false);   // the tile split does not change the workspace
    if (pp.use)
        return std::max(pp.conv_bytes,
                        plan_sk(g, pp, q->type, p->causal, p->scale, p->logit_softcap, sms).bytes());
    return plan_split(g, sms, g.n_kv, false).part_bytes;
}

int launch_encoder_sk(const SkPlan &sp, const CUtensorMap &mk, const CUtensorMap &mv, const CUtensorMap &mq,
                      const CUtensorMap &mo, const PrefillArgs &a, void *workspace, cudaStream_t st) {
    using C = SkCfg<64>;
    static std::atomic<int> attr_done[kMaxDevices];
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_done[dev].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(fa_encoder_sk_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
            cudaSuccess)
            return VTX_ERR_CUDA;
        attr_done[dev].store(1, std::memory_order_release);
    }
    char *ws = static_cast<char *>(workspace);
    SkArgs sk{};
    sk.n_pairs = sp.n_pairs;
    sk.n_iter = sp.n_iter;
    sk.total = sp.total;
    std::memcpy(sk.bound, sp.bound, sizeof(int) * (sp.ctas + 1));
    sk.flags = reinterpret_cast<unsigned long long *>(ws);
    float *part = reinterpret_cast<float *>(ws + sp.flags_bytes);
    sk.part = part;
    CUtensorMap mp;
    const int rc = encode_part_map(&mp, part, 2 * sp.ctas);
    if (rc != VTX_OK) return rc;
    return launch_pdl(fa_encoder_sk_kernel<64>, dim3((unsigned)sp.ctas), dim3(C::NTHREADS), C::SMEM, st, mk, mv, mq,
                      mo, mp, a, sk);
}

// The batched ragged decode shared by vtx_flash_attn_decode_batched (scratch =
// the caller's workspace) and vtx_flash_attn_decode_batched_noalloc (scratch =
// the library's built-in buffer, looked up through get_scratch once the batch
// is known to fit).  too_big is the status returned when the split partials do
// not fit in scratch_bytes.
int decode_batched_impl(const vtx_decode_batch *b, void *scratch, size_t scratch_bytes, cudaStream_t st, int too_big,
                        int (*get_scratch)(void **)) {
    if (!b) return VTX_ERR_NULL;
    if (b->n_seq < 0 || b->n_head_q <= 0 || b->n_head_kv <= 0 || b->n_head_q % b->n_head_kv || b->max_kv_len < 0)
        return VTX_ERR_SHAPE;
    if (b->head_dim != 64 && b->head_dim != 128) return VTX_ERR_UNSUPPORTED;
    if (b->kv_type != VTX_TYPE_F16 && b->kv_type != VTX_TYPE_F32 && b->kv_type != VTX_TYPE_Q8_0) return VTX_ERR_TYPE;
    if (b->n_seq == 0) return VTX_OK;
    if (!b->q || !b->k_ptrs || !b->v_ptrs || !b->kv_len || !b->dst) return VTX_ERR_NULL;
    if (b->n_seq > 65535 || b->n_head_q / b->n_head_kv > 16) return VTX_ERR_UNSUPPORTED;
    DeviceState *ds = nullptr;
    int rc = ensure_device(&ds);
    if (rc != VTX_OK) return rc;
    const int D = b->head_dim;
    Geo g{D, 1, std::max(1, b->max_kv_len), b->n_head_q, b->n_head_kv, b->n_head_q / b->n_head_kv, b->n_seq,
          b->n_seq, b->kv_type};
    const SplitPlan sp = plan_split(g, ds->sms, g.n_kv, true, batch_streaming(b), batch_q8_ctas(b));
    if (scratch_bytes < sp.part_bytes) return too_big;
    if (get_scratch && sp.part_bytes) {
        rc = get_scratch(&scratch);
        if (rc != VTX_OK) return rc;
    }
    if (scratch && reinterpret_cast<uintptr_t>(scratch) % 256) return VTX_ERR_WORKSPACE;
    SplitArgs a{};
    a.q = reinterpret_cast<const char *>(b->q);
    a.q_nb1 = (long long)b->n_head_q * D * 4; a.q_nb2 = (long long)D * 4; a.q_nb3 = (long long)b->n_head_q * D * 4;
    a.k_ptrs = b->k_ptrs; a.v_ptrs = b->v_ptrs; a.kv_len = b->kv_len; a.fresh = b->fresh_row;
    a.k_nb1 = a.v_nb1 = (long long)b->kv_nb1;
    a.k_nb2 = a.v_nb2 = (long long)b->kv_nb2;
    a.k_bdiv = a.v_bdiv = 1;
    a.n_kv = g.n_kv;
    a.dst = reinterpret_cast<char *>(b->dst);
    a.d_nb1 = (long long)D * 4; a.d_nb2 = (long long)b->n_head_q * D * 4; a.d_nb3 = (long long)b->n_head_q * D * 4;
    a.n_q = 1; a.Hq = b->n_head_q; a.Hkv = b->n_head_kv; a.G = g.G; a.B = b->n_seq;
    a.tok_per_cta = sp.tok_per_cta; a.hc = sp.hc; a.n_hchunks = sp.n_hchunks; a.n_qtiles = sp.n_qtiles;
    a.chunk = sp.chunk; a.n_splits = sp.n_splits;
    float qk_scale, softcap, m0, m1;
    int nhl2;
    fill_math(b->scale, 0.0f, 0.0f, b->n_head_q, &qk_scale, &softcap, &m0, &m1, &nhl2);
    a.qk_scale = qk_scale; a.softcap = 0.0f; a.max_bias = 0.0f; a.m0 = m0; a.m1 = m1; a.n_head_log2 = nhl2;
    a.write_final = sp.n_splits <= 1;
    if (!a.write_final) {
        const size_t work = (size_t)g.B * g.Hkv * sp.n_hchunks * sp.n_qtiles * sp.n_splits * sp.maxr;
        a.part_o = static_cast<float *>(scratch);
        a.part_ml = reinterpret_cast<float *>(static_cast<char *>(scratch) + align_up(work * D * 4, 256));
    }
    const int rb = row_bytes(b->kv_type, D);
    a.vec = pick_vec(rb, {(unsigned long long)b->kv_nb1, (unsigned long long)(b->n_head_kv > 1 ? b->kv_nb2 : 0)});
    // stream base pointers are only known on the device: require 16-byte
    // aligned bases whenever the strides allow 16-byte copies
    if (!a.vec) return VTX_ERR_STRIDE;
    a.err = ds->err;
    if (decode_mma_ok(b->kv_type, 1, g.G, a.vec, sp.maxr, sp.n_hchunks)) return launch_decode_mma(a, D, st);
    if (decode_f32_ok(b->kv_type, 1, g.G, a.vec, sp.maxr, sp.n_hchunks)) return launch_decode_f32(a, D, st);
    if (const int hpc = decode_q8_hpc(b->kv_type, D, 1, g.G, g.Hkv, sp.maxr, sp.n_hchunks, a.k_nb1, a.k_nb2,
                                      a.v_nb1, a.v_nb2))
        return launch_decode_q8(a, hpc, st);
    dim3 grid((unsigned)sp.n_splits, (unsigned)(g.Hkv * sp.n_hchunks), (unsigned)b->n_seq);
    return launch_split(a, D, b->kv_type, sp.maxr, grid, st);
}

// Fused decode layer (decode_layer.cuh): splits per (stream, KV head) so one
// wave covers the GPU, at least one 16-key tile per warp; workspace = the
// split partials (O, then (m, l)) and one arrival counter per (stream, KV
// head), which must be zero before the first call (every call leaves it so).
// With the cluster merge (`cluster` > 1) the splits of a (stream, KV head) are
// the CTAs of one cluster and the workspace is not used; its size is that of
// the global merge either way, so the workspace query needs no device.
struct LayerPlan {
    int n_splits = 1;
    int cluster = 0;                            // > 1: splits per cluster (= the launch's n_splits)
    size_t o_bytes = 0, ml_bytes = 0, flag_bytes = 0, bytes = 0;
};

// Clusters of cs CTAs (cs = 1..8) of the decode-layer kernel of one cache
// type that can be resident at once on the current device (one CTA per SM:
// its shared memory), queried once per device.
struct LayerClusters {
    int max_active[LayerCfg<1>::CLMAX + 1];
};

template <int KVT>
const LayerClusters *layer_clusters() {
    using C = LayerCfg<KVT>;
    static std::atomic<int> ready[kMaxDevices];              // 0 not yet, 1 done, 2 unavailable
    static LayerClusters tab[kMaxDevices];
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    int st = ready[dev].load(std::memory_order_acquire);
    if (st == 0) {
        std::lock_guard<std::mutex> lk(mu);
        st = ready[dev].load(std::memory_order_relaxed);
        if (st == 0) {
            bool ok = cudaFuncSetAttribute(fa_decode_layer_kernel<KVT, true>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) == cudaSuccess;
            LayerClusters t{};
            for (int cs = 1; ok && cs <= C::CLMAX; ++cs) {
                cudaLaunchConfig_t cfg = {};
                cfg.gridDim = dim3((unsigned)cs);
                cfg.blockDim = dim3(C::NT);
                cfg.dynamicSmemBytes = C::SMEM;
                cudaLaunchAttribute attr[1];
                attr[0].id = cudaLaunchAttributeClusterDimension;
                attr[0].val.clusterDim.x = (unsigned)cs;
                attr[0].val.clusterDim.y = 1;
                attr[0].val.clusterDim.z = 1;
                cfg.attrs = attr;
                cfg.numAttrs = 1;
                ok = cudaOccupancyMaxActiveClusters(&t.max_active[cs], fa_decode_layer_kernel<KVT, true>, &cfg) ==
                     cudaSuccess;
            }
            if (ok) tab[dev] = t;
            else cudaGetLastError();
            st = ok ? 1 : 2;
            ready[dev].store(st, std::memory_order_release);
        }
    }
    return st == 1 ? &tab[dev] : nullptr;
}

int check_layer_args(const vtx_decode_layer_args *p) {
    if (!p) return VTX_ERR_NULL;
    if (p->n_seq < 0 || p->n_head_q <= 0 || p->n_head_kv <= 0 || p->n_head_q % p->n_head_kv || p->max_kv_len < 0)
        return VTX_ERR_SHAPE;
    if (p->head_dim != 128 || p->n_head_q / p->n_head_kv > 8) return VTX_ERR_UNSUPPORTED;
    if (p->kv_type != VTX_TYPE_F16 && p->kv_type != VTX_TYPE_Q8_0) return VTX_ERR_TYPE;
    if (p->kv_type == VTX_TYPE_Q8_0 && p->n_head_kv % 2) return VTX_ERR_UNSUPPORTED;
    if (!(p->freq_base > 0.0f)) return VTX_ERR_SHAPE;
    if ((long long)p->n_seq * p->n_head_kv > (1LL << 24)) return VTX_ERR_UNSUPPORTED;
    return VTX_OK;
}

// Splits per (stream, KV head): enough for one wave over the SMs, at most one
// per W tiles of max_kv_len.  With a cluster table: when that is at most
// twice the largest cluster size cs whose clusters (one per (stream, KV head))
// fit twice over -- this launch's and the next layer's, which then becomes
// resident and streams its ring early -- the splits are min(splits, cs) CTAs
// of one cluster, merged through distributed shared memory; otherwise the
// global merge.  Measured on B200 (batch 1, 8 KV heads, graph replay, us per
// layer, global / cluster of 6): F16 391 keys 5.70 / 4.28, 600 keys 6.01 /
// 4.48; Q8_0 800 keys 7.78 / 6.35, 2000 keys 8.30 / 7.65; at 7300 Q8_0 keys
// (18 splits) 11.56 / 16.32.
LayerPlan plan_layer(const vtx_decode_layer_args *p, int sms, const LayerClusters *cl = nullptr) {
    LayerPlan lp;
    const long long items = (long long)p->n_seq * p->n_head_kv;
    const int tiles = (std::max(1, p->max_kv_len) + 15) / 16;
    const int minb = p->kv_type == VTX_TYPE_Q8_0 ? LayerCfg<8>::MINB : LayerCfg<1>::MINB;   // CTAs per SM
    const long long by_wave = std::max<long long>(1, (long long)sms * minb / std::max<long long>(1, items));
    const int w = p->kv_type == VTX_TYPE_Q8_0 ? LayerCfg<8>::W : LayerCfg<1>::W;           // warps per CTA
    lp.n_splits = (int)std::max<long long>(1, std::min<long long>(by_wave, (tiles + w - 1) / w));
    const int G = p->n_head_q / p->n_head_kv;
    if (lp.n_splits > 1) {
        const size_t rows = (size_t)items * lp.n_splits * G;
        lp.o_bytes = align_up(rows * p->head_dim * 4, 256);
        lp.ml_bytes = align_up(rows * 8, 256);
        lp.flag_bytes = align_up((size_t)items * 4, 256);
        if (cl) {
            int fit = 0;
            for (int cs = 2; cs <= LayerCfg<1>::CLMAX; ++cs)
                if (cl->max_active[cs] >= 2 * items) fit = cs;
            if (fit >= 2 && lp.n_splits <= 2 * fit) lp.cluster = std::min(lp.n_splits, fit);
        }
    }
    lp.bytes = lp.o_bytes + lp.ml_bytes + lp.flag_bytes;
    return lp;
}

template <int KVT>
int launch_decode_layer_t(const DecodeLayerArgs &a, unsigned ctas, int cluster, cudaStream_t st) {
    using C = LayerCfg<KVT>;
    if (cluster > 1)                            // attribute set by layer_clusters()
        return launch_pdl_cluster(fa_decode_layer_kernel<KVT, true>, dim3(ctas), dim3(C::NT), C::SMEM, st, cluster,
                                  a);
    static std::atomic<int> attr_done[kMaxDevices];
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_done[dev].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(fa_decode_layer_kernel<KVT, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 C::SMEM) != cudaSuccess)
            return VTX_ERR_CUDA;
        attr_done[dev].store(1, std::memory_order_release);
    }
    return launch_pdl(fa_decode_layer_kernel<KVT, false>, dim3(ctas), dim3(C::NT), C::SMEM, st, a);
}

}  // namespace

// ================================================================================
extern "C" {

const char *vtx_strerror(int status) {
    switch (status) {
        case VTX_OK: return "ok";
        case VTX_ERR_NULL: return "required pointer is NULL";
        case VTX_ERR_TYPE: return "unsupported or mismatched tensor type";
        case VTX_ERR_SHAPE: return "inconsistent tensor shapes";
        case VTX_ERR_STRIDE: return "unsupported stride or alignment";
        case VTX_ERR_UNSUPPORTED: return "unsupported head_dim or parameter";
        case VTX_ERR_WORKSPACE: return "workspace too small or misaligned";
        case VTX_ERR_CUDA: return "CUDA launch or runtime call failed";
        case VTX_ERR_NO_DEVICE: return "no sm_100 device is current";
        case VTX_ERR_SCRATCH_LIMIT: return "problem needs more scratch than the built-in no-alloc buffer holds";
        default: return "unknown status";
    }
}

int vtx_abi_version(void) { return VTX_FA_ABI_VERSION; }

size_t vtx_flash_attn_ext_workspace(const vtx_tensor *q, const vtx_tensor *k, const vtx_tensor *v,
                                    const vtx_fa_params *params) {
    Geo g;
    if (check_operands(q, k, v, nullptr, params, nullptr, &g) != VTX_OK) return (size_t)-1;
    int sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaGetLastError();
    return workspace_for(g, q, k, v, params, sms);
}

int vtx_flash_attn_ext(const vtx_tensor *q, const vtx_tensor *k, const vtx_tensor *v, const vtx_tensor *mask,
                       const vtx_fa_params *params, vtx_tensor *dst, void *workspace, size_t workspace_bytes,
                       void *stream) {
    if (!dst) return VTX_ERR_NULL;
    Geo g;
    int rc = check_operands(q, k, v, mask, params, dst, &g);
    if (rc != VTX_OK) return rc;
    if ((g.n_q > 0 && g.n_kv > 0) && (!q->data || !k->data || !v->data || !dst->data)) return VTX_ERR_NULL;
    if (mask && !mask->data) return VTX_ERR_NULL;
    if (reinterpret_cast<uintptr_t>(dst->data) % 16) return VTX_ERR_STRIDE;
    DeviceState *ds = nullptr;
    rc = ensure_device(&ds);
    if (rc != VTX_OK) return rc;
    if (g.n_q == 0 || g.B == 0 || g.Hq == 0) return VTX_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (workspace_bytes < workspace_for(g, q, k, v, params, ds->sms)) return VTX_ERR_WORKSPACE;
    if (workspace && reinterpret_cast<uintptr_t>(workspace) % 256) return VTX_ERR_WORKSPACE;

    float qk_scale, softcap, m0, m1;
    int nhl2;
    fill_math(params->scale, params->max_bias, params->logit_softcap, g.Hq, &qk_scale, &softcap, &m0, &m1, &nhl2);

    const PrefillPlan pp = plan_prefill(g, q, k, v, ds->sms, params->causal != 0);
    if (pp.use && g.n_kv > 0) {
        const void *kp = k->data, *vp = v->data;
        size_t knb1 = k->nb[1], knb2 = k->nb[2], knb3 = k->nb[3];
        size_t vnb1 = v->nb[1], vnb2 = v->nb[2], vnb3 = v->nb[3];
        if (pp.convert) {
            __half *kc = static_cast<__half *>(workspace);
            __half *vc = reinterpret_cast<__half *>(static_cast<char *>(workspace) + pp.conv_bytes / 2);
            const long long total = (long long)g.Bkv * g.Hkv * g.n_kv * g.D;
            const int blocks = (int)std::min<long long>((total + 255) / 256, 8LL * ds->sms);
            if (launch_pdl(convert_kv_f16_kernel, dim3(blocks), dim3(256), 0, st, static_cast<const char *>(k->data),
                           (long long)k->nb[1], (long long)k->nb[2], (long long)k->nb[3], (int)k->type, g.D, g.n_kv,
                           g.Hkv, g.Bkv, kc) != VTX_OK ||
                launch_pdl(convert_kv_f16_kernel, dim3(blocks), dim3(256), 0, st, static_cast<const char *>(v->data),
                           (long long)v->nb[1], (long long)v->nb[2], (long long)v->nb[3], (int)v->type, g.D, g.n_kv,
                           g.Hkv, g.Bkv, vc) != VTX_OK)
                return VTX_ERR_CUDA;
            kp = kc;
            vp = vc;
            knb1 = vnb1 = (size_t)g.D * 2;
            knb2 = vnb2 = knb1 * g.n_kv;
            knb3 = vnb3 = knb2 * g.Hkv;
        }
        CUtensorMap mk, mv;
        rc = encode_kv_map(&mk, kp, g.D, g.n_kv, g.Hkv, g.Bkv, knb1, knb2, knb3);
        if (rc != VTX_OK) return rc;
        rc = encode_kv_map(&mv, vp, g.D, g.n_kv, g.Hkv, g.Bkv, vnb1, vnb2, vnb3);
        if (rc != VTX_OK) return rc;
        PrefillArgs a{};
        a.q = static_cast<const char *>(q->data);
        a.q_f16 = q->type == VTX_TYPE_F16;
        a.q_nb1 = (long long)q->nb[1]; a.q_nb2 = (long long)q->nb[2]; a.q_nb3 = (long long)q->nb[3];
        if (mask) {
            a.mask = static_cast<const char *>(mask->data);
            a.m_nb1 = (long long)mask->nb[1]; a.m_nb2 = (long long)mask->nb[2]; a.m_nb3 = (long long)mask->nb[3];
            a.m_ne2 = (int)mask->ne[2]; a.m_ne3 = (int)mask->ne[3];
        }
        a.dst = static_cast<char *>(dst->data);
        a.d_nb1 = (long long)dst->nb[1]; a.d_nb2 = (long long)dst->nb[2]; a.d_nb3 = (long long)dst->nb[3];
        a.n_q = g.n_q; a.n_kv = g.n_kv; a.Hq = g.Hq; a.Hkv = g.Hkv; a.G = g.G; a.B = g.B;
        a.tok_per_tile = pp.tok_per_tile; a.n_tiles_q = pp.n_tiles_q; a.n_cta_q = pp.n_cta_q;
        a.kv_bdiv = g.B / g.Bkv;
        a.fused = (softcap == 0.0f && params->scale > 0.0f) ? 1 : 0;
        a.cx = a.fused ? params->scale * kLog2e : kLog2e;
        a.qk_scale = qk_scale; a.softcap = softcap; a.scale = params->scale;
        a.max_bias = params->max_bias; a.m0 = m0; a.m1 = m1; a.n_head_log2 = nhl2;
        a.causal = params->causal; a.window = params->window;
        a.q_quant8 = g.kv_type == VTX_TYPE_Q8_0;
        a.err = ds->err;
        CUtensorMap mo;
        std::memset(&mo, 0, sizeof(mo));
        a.o_f16 = dst->type == VTX_TYPE_F16;
        a.o_tma = encode_out_map(&mo, dst->data, g.D, g.Hq, g.n_q, g.B, dst->nb[1], dst->nb[2], dst->nb[3], g.G,
                                 pp.tok_per_tile, a.o_f16) == VTX_OK;
        if (a.o_f16 && !a.o_tma) return VTX_ERR_STRIDE;       // F16 results leave by the TMA epilogue only
        CUtensorMap mq;
        std::memset(&mq, 0, sizeof(mq));
        a.q_tma = q->type == VTX_TYPE_F16 && !a.q_quant8 &&
                  encode_q_map(&mq, q->data, g.D, g.Hq, g.n_q, g.B, q->nb[1], q->nb[2], q->nb[3], g.G,
                               pp.tok_per_tile) == VTX_OK;
        if (!mask && a.q_tma && a.o_tma && !a.o_f16) {
            const SkPlan sp =
                plan_sk_ranges(g, pp, q->type, params->causal, params->scale, params->logit_softcap, ds->sms);
            if (sp.use) {
                if (!workspace) return VTX_ERR_WORKSPACE;
                return launch_encoder_sk(sp, mk, mv, mq, mo, a, workspace, st);
            }
        }
        if ((long long)pp.n_cta_q * g.Hkv > 0x7fffffffLL) return VTX_ERR_UNSUPPORTED;
        // causal launches without a mask tensor or softcap, windowed or of more
        // than one wave, run the causal instantiation; beyond one wave its CTAs
        // go longest first (see the kernel)
        a.lpt = params->causal && !mask && a.fused && (long long)pp.n_cta_q * g.Hkv * g.B > ds->sms;
        const dim3 grid = a.lpt ? dim3((unsigned)(pp.n_cta_q * g.Hkv), 1, g.B) : dim3(pp.n_cta_q, g.Hkv, g.B);
        return launch_prefill(g.D, pp.nqt, mask != nullptr, mk, mv, mo, mq, a, grid, st);
    }

    // F16 results come only from the tcgen05 kernel's TMA epilogue (above)
    if (dst->type != VTX_TYPE_F32) return VTX_ERR_TYPE;

    // ---- split-KV path ---------------------------------------------------------
    const SplitPlan sp = plan_split(g, ds->sms, g.n_kv, false);
    SplitArgs a{};
    a.q = static_cast<const char *>(q->data);
    a.q_f16 = q->type == VTX_TYPE_F16;
    a.q_nb1 = (long long)q->nb[1]; a.q_nb2 = (long long)q->nb[2]; a.q_nb3 = (long long)q->nb[3];
    a.k = static_cast<const char *>(k->data); a.v = static_cast<const char *>(v->data);
    a.k_nb1 = (long long)k->nb[1]; a.k_nb2 = (long long)k->nb[2]; a.k_nb3 = (long long)k->nb[3];
    a.v_nb1 = (long long)v->nb[1]; a.v_nb2 = (long long)v->nb[2]; a.v_nb3 = (long long)v->nb[3];
    a.k_bdiv = g.B / g.Bkv; a.v_bdiv = g.B / g.Bkv;
    a.n_kv = g.n_kv;
    if (mask) {
        a.mask = static_cast<const char *>(mask->data);
        a.m_nb1 = (long long)mask->nb[1]; a.m_nb2 = (long long)mask->nb[2]; a.m_nb3 = (long long)mask->nb[3];
        a.m_ne2 = (int)mask->ne[2]; a.m_ne3 = (int)mask->ne[3];
    }
    a.dst = static_cast<char *>(dst->data);
    a.d_nb1 = (long long)dst->nb[1]; a.d_nb2 = (long long)dst->nb[2]; a.d_nb3 = (long long)dst->nb[3];
    a.n_q = g.n_q; a.Hq = g.Hq; a.Hkv = g.Hkv; a.G = g.G; a.B = g.B;
    a.tok_per_cta = sp.tok_per_cta; a.hc = sp.hc; a.n_hchunks = sp.n_hchunks; a.n_qtiles = sp.n_qtiles;
    a.chunk = sp.chunk; a.n_splits = sp.n_splits;
    a.qk_scale = qk_scale; a.softcap = softcap; a.max_bias = params->max_bias; a.m0 = m0; a.m1 = m1;
    a.n_head_log2 = nhl2;
    a.causal = params->causal; a.window = params->window;
    a.write_final = sp.n_splits <= 1;
    if (!a.write_final) {
        const size_t work = (size_t)g.B * g.Hkv * sp.n_hchunks * sp.n_qtiles * sp.n_splits * sp.maxr;
        a.part_o = static_cast<float *>(workspace);
        a.part_ml = reinterpret_cast<float *>(static_cast<char *>(workspace) + align_up(work * g.D * 4, 256));
    }
    const int rb = row_bytes(g.kv_type, g.D);
    a.vec = pick_vec(rb, {reinterpret_cast<uintptr_t>(k->data), reinterpret_cast<uintptr_t>(v->data),
                          (unsigned long long)k->nb[1], (unsigned long long)(g.Hkv > 1 ? k->nb[2] : 0),
                          (unsigned long long)(g.Bkv > 1 ? k->nb[3] : 0), (unsigned long long)v->nb[1],
                          (unsigned long long)(g.Hkv > 1 ? v->nb[2] : 0),
                          (unsigned long long)(g.Bkv > 1 ? v->nb[3] : 0)});
    if (!a.vec) return VTX_ERR_STRIDE;
    a.err = ds->err;
    if (decode_mma_ok(g.kv_type, g.n_q, g.G, a.vec, sp.maxr, sp.n_hchunks) && !mask && !params->causal &&
        params->logit_softcap == 0.0f)
        return launch_decode_mma(a, g.D, st);
    if (decode_f32_ok(g.kv_type, g.n_q, g.G, a.vec, sp.maxr, sp.n_hchunks) && !mask && !params->causal &&
        params->logit_softcap == 0.0f)
        return launch_decode_f32(a, g.D, st);
    if (!mask && !params->causal && params->logit_softcap == 0.0f) {
        const int hpc = decode_q8_hpc(g.kv_type, g.D, g.n_q, g.G, g.Hkv, sp.maxr, sp.n_hchunks, a.k_nb1, a.k_nb2,
                                      a.v_nb1, a.v_nb2);
        const uintptr_t bases = reinterpret_cast<uintptr_t>(a.k) | reinterpret_cast<uintptr_t>(a.v) |
                                (uintptr_t)a.k_nb3 | (uintptr_t)a.v_nb3;
        if (hpc && bases % 16 == 0) return launch_decode_q8(a, hpc, st);
    }
    dim3 grid((unsigned)(sp.n_splits * sp.n_qtiles), (unsigned)(g.Hkv * sp.n_hchunks), (unsigned)g.B);
    return launch_split(a, g.D, g.kv_type, sp.maxr, grid, st);
}

size_t vtx_flash_attn_decode_batched_workspace(const vtx_decode_batch *b) {
    if (!b || b->n_seq < 0 || b->n_head_kv <= 0 || b->n_head_q % b->n_head_kv) return (size_t)-1;
    if (b->head_dim != 64 && b->head_dim != 128) return (size_t)-1;
    Geo g{b->head_dim, 1, std::max(1, b->max_kv_len), b->n_head_q, b->n_head_kv, b->n_head_q / b->n_head_kv,
          b->n_seq, b->n_seq, b->kv_type};
    int sms = 148, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaGetLastError();
    return plan_split(g, sms, g.n_kv, true, batch_streaming(b), batch_q8_ctas(b)).part_bytes;
}

int vtx_flash_attn_decode_batched(const vtx_decode_batch *b, void *workspace, size_t workspace_bytes, void *stream) {
    return decode_batched_impl(b, workspace, workspace_bytes, static_cast<cudaStream_t>(stream), VTX_ERR_WORKSPACE,
                               nullptr);
}

int vtx_kv_append(const vtx_kv_append_args *p, void *stream) {
    if (!p) return VTX_ERR_NULL;
    if (p->n_tokens < 0 || p->n_head_kv <= 0 || p->n_head_q < 0) return VTX_ERR_SHAPE;
    if (p->head_dim != 64 && p->head_dim != 128) return VTX_ERR_UNSUPPORTED;
    if (p->kv_type != VTX_TYPE_F32 && p->kv_type != VTX_TYPE_F16 && p->kv_type != VTX_TYPE_Q8_0) return VTX_ERR_TYPE;
    if (p->n_tokens == 0) return VTX_OK;
    if (!p->k || !p->v || !p->positions || !p->slots) return VTX_ERR_NULL;
    if ((!p->k_cache && !p->k_cache_ptrs) || (!p->v_cache && !p->v_cache_ptrs)) return VTX_ERR_NULL;
    if (p->q_out && (!p->q || p->n_head_q <= 0)) return VTX_ERR_NULL;
    if (!(p->freq_base > 0.0f)) return VTX_ERR_SHAPE;
    if ((long long)p->n_head_q + 2LL * p->n_head_kv > 8LL * 65535) return VTX_ERR_UNSUPPORTED;   // grid.y
    // float2 row loads / stores; half2 (F16) or 2-byte (Q8_0) cache stores
    const uintptr_t rows = reinterpret_cast<uintptr_t>(p->k) | reinterpret_cast<uintptr_t>(p->v) | p->k_nb1 |
                           p->v_nb1 | (p->q_out ? reinterpret_cast<uintptr_t>(p->q) | reinterpret_cast<uintptr_t>(p->q_out) |
                                                      p->q_nb1 | p->q_out_nb1
                                                : 0);
    const uintptr_t cache = reinterpret_cast<uintptr_t>(p->k_cache) | reinterpret_cast<uintptr_t>(p->v_cache) |
                            p->cache_nb1;
    const unsigned calign = p->kv_type == VTX_TYPE_F32 ? 8 : p->kv_type == VTX_TYPE_F16 ? 4 : 2;
    if (rows % 8 || cache % calign) return VTX_ERR_STRIDE;
    DeviceState *ds = nullptr;
    int rc = ensure_device(&ds);
    if (rc != VTX_OK) return rc;
    KvAppendArgs a{};
    a.T = p->n_tokens; a.Hq = p->q_out ? p->n_head_q : 0; a.Hkv = p->n_head_kv; a.kv_type = p->kv_type;
    a.theta_scale = std::pow(p->freq_base, -2.0f / (float)p->head_dim);   // as ggml: powf on the host
    a.q = p->q; a.q_nb1 = (long long)(p->q_nb1 / 4);
    a.q_out = p->q_out; a.qo_nb1 = (long long)(p->q_out_nb1 / 4);
    a.k = p->k; a.k_nb1 = (long long)(p->k_nb1 / 4);
    a.v = p->v; a.v_nb1 = (long long)(p->v_nb1 / 4);
    a.positions = p->positions; a.slots = p->slots;
    a.k_cache = static_cast<char *>(p->k_cache); a.v_cache = static_cast<char *>(p->v_cache);
    a.k_ptrs = p->k_cache_ptrs; a.v_ptrs = p->v_cache_ptrs;
    a.cache_nb1 = (long long)p->cache_nb1;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // a decode step's few tokens: 8 rows (one per warp) per CTA, so the rows are
    // in flight together; many tokens: one CTA per token, one table build each
    const int per_tok = a.Hq + 2 * a.Hkv;
    a.rows_per_cta = a.T >= 2 * ds->sms ? per_tok : 8;
    const dim3 grid((unsigned)a.T, (unsigned)((per_tok + a.rows_per_cta - 1) / a.rows_per_cta));
    return p->head_dim == 64 ? launch_pdl(kv_append_kernel<64>, grid, dim3(256), 0, st, a)
                             : launch_pdl(kv_append_kernel<128>, grid, dim3(256), 0, st, a);
}

int vtx_decode_advance(int32_t *positions, int32_t *slots, int32_t *kv_len, int32_t n, int32_t window,
                       void *stream) {
    if (n < 0 || window <= 0) return VTX_ERR_SHAPE;
    if (n == 0 || (!positions && !slots && !kv_len)) return VTX_OK;
    DeviceState *ds = nullptr;
    int rc = ensure_device(&ds);
    if (rc != VTX_OK) return rc;
    return launch_pdl(decode_advance_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0,
                      static_cast<cudaStream_t>(stream), positions, slots, kv_len, (int)n, (int)window);
}

size_t vtx_decode_layer_workspace(const vtx_decode_layer_args *p) {
    if (check_layer_args(p) != VTX_OK) return (size_t)-1;
    int sms = 148, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaGetLastError();
    return plan_layer(p, sms).bytes;
}

int vtx_decode_layer(const vtx_decode_layer_args *p, void *workspace, size_t workspace_bytes, void *stream) {
    int rc = check_layer_args(p);
    if (rc != VTX_OK) return rc;
    if (p->n_seq == 0) return VTX_OK;
    if (!p->q || !p->k || !p->v || !p->dst || !p->positions || !p->slots || !p->kv_len || !p->k_cache_ptrs ||
        !p->v_cache_ptrs)
        return VTX_ERR_NULL;
    const uintptr_t al = reinterpret_cast<uintptr_t>(p->q) | reinterpret_cast<uintptr_t>(p->k) |
                         reinterpret_cast<uintptr_t>(p->v) | reinterpret_cast<uintptr_t>(p->dst) | p->q_nb1 |
                         p->k_nb1 | p->v_nb1 | p->dst_nb1 | p->cache_nb1;
    if (al % 16) return VTX_ERR_STRIDE;
    const size_t hb = p->kv_type == VTX_TYPE_Q8_0 ? (size_t)p->head_dim / 32 * 34 : (size_t)p->head_dim * 2;
    if (p->cache_nb1 < hb * p->n_head_kv) return VTX_ERR_STRIDE;
    DeviceState *ds = nullptr;
    rc = ensure_device(&ds);
    if (rc != VTX_OK) return rc;
    const LayerClusters *cl = p->kv_type == VTX_TYPE_F16 ? layer_clusters<1>() : layer_clusters<8>();
    const LayerPlan lp = plan_layer(p, ds->sms, cl);
    if (workspace_bytes < lp.bytes) return VTX_ERR_WORKSPACE;
    if (lp.bytes && (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256)) return VTX_ERR_WORKSPACE;
    DecodeLayerArgs a{};
    a.n_seq = p->n_seq; a.Hq = p->n_head_q; a.Hkv = p->n_head_kv; a.G = p->n_head_q / p->n_head_kv;
    a.q = p->q; a.k = p->k; a.v = p->v;
    a.q_nb1 = (long long)(p->q_nb1 / 4); a.k_nb1 = (long long)(p->k_nb1 / 4); a.v_nb1 = (long long)(p->v_nb1 / 4);
    a.positions = p->positions; a.slots = p->slots; a.kv_len = p->kv_len;
    a.k_ptrs = p->k_cache_ptrs; a.v_ptrs = p->v_cache_ptrs;
    a.cache_nb1 = (long long)p->cache_nb1;
    a.theta_scale = std::pow(p->freq_base, -2.0f / (float)p->head_dim);   // as ggml: powf on the host
    a.cx = p->scale * kLog2e;
    a.dst = p->dst; a.dst_nb1 = (long long)(p->dst_nb1 / 4);
    a.n_splits = lp.cluster > 1 ? lp.cluster : lp.n_splits;
    char *ws = static_cast<char *>(workspace);
    if (lp.bytes && lp.cluster <= 1) {
        a.part_o = reinterpret_cast<float *>(ws);
        a.part_ml = reinterpret_cast<float *>(ws + lp.o_bytes);
        a.flags = reinterpret_cast<unsigned *>(ws + lp.o_bytes + lp.ml_bytes);
    }
    a.early = p->early ? 1 : 0;
    a.err = ds->err;
    const unsigned ctas = (unsigned)((long long)p->n_seq * p->n_head_kv * a.n_splits);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return p->kv_type == VTX_TYPE_F16 ? launch_decode_layer_t<1>(a, ctas, lp.cluster, st)
                                      : launch_decode_layer_t<8>(a, ctas, lp.cluster, st);
}

int vtx_encoder_chunk_plan(int32_t total_mel_frames, vtx_enc_chunk *chunks, int32_t max_chunks,
                           int32_t *n_tokens_total, int32_t *n_tokens_used) {
    if (total_mel_frames < 0 || max_chunks < 0) return VTX_ERR_SHAPE;
    if (!chunks && max_chunks > 0) return VTX_ERR_NULL;
    // the walk of run_encoder_chunked (src/voxtral.cpp:2234-2335)
    const int alloc_total = enc_tokens_total(total_mel_frames);
    const int stride_mel = kEncChunkMel - 2 * kEncChunkOverlap;
    int n = 0, write = 0;
    for (int off = 0; alloc_total > 0 && off < total_mel_frames; off += stride_mel) {
        const int frames = std::min(kEncChunkMel, total_mel_frames - off);
        const int skip = n > 0 ? kEncChunkOverlap : 0;
        const int toks = enc_tokens_of(frames);
        int stride = toks - skip;
        if (stride <= 0) break;                                   // no new tokens: stop (:2265-2272, :2300-2305)
        if (write + stride > alloc_total) {                       // clamp to the allocation (:2307-2311)
            stride = alloc_total - write;
            if (stride <= 0) break;
        }
        if (n < max_chunks) {
            vtx_enc_chunk &c = chunks[n];
            c.mel_offset = off; c.mel_frames = frames; c.n_tokens = toks; c.skip = skip; c.stride = stride;
            c.rope_offset = write - skip; c.write_offset = write; c.reserved = 0;
        }
        write += stride;
        ++n;
    }
    if (n_tokens_total) *n_tokens_total = std::max(alloc_total, 0);
    if (n_tokens_used) *n_tokens_used = write / kEncDownsample * kEncDownsample;
    return n;
}

int vtx_encoder_stitch(const void *src, size_t src_chunk_bytes, size_t src_row_bytes, void *dst,
                       size_t dst_row_bytes, size_t row_bytes, const vtx_enc_chunk *chunks, int32_t n_chunks,
                       void *stream) {
    if (n_chunks < 0) return VTX_ERR_SHAPE;
    if (n_chunks == 0 || row_bytes == 0) return VTX_OK;
    if (!src || !dst || !chunks) return VTX_ERR_NULL;
    long long rows = 0;
    for (int c = 0; c < n_chunks; ++c) {
        const vtx_enc_chunk &ch = chunks[c];
        if (ch.skip < 0 || ch.stride < 0 || ch.write_offset < 0) return VTX_ERR_SHAPE;
        rows += ch.stride;
    }
    if (rows > 0x7fffffffLL) return VTX_ERR_UNSUPPORTED;
    DeviceState *ds = nullptr;
    int rc = ensure_device(&ds);
    if (rc != VTX_OK) return rc;
    const uintptr_t al = reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | src_chunk_bytes |
                         src_row_bytes | dst_row_bytes | row_bytes;
    const int vec = al % 16 == 0 ? 16 : al % 8 == 0 ? 8 : al % 4 == 0 ? 4 : 1;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    for (int c0 = 0; c0 < n_chunks; c0 += kStitchMaxChunks) {
        StitchArgs a{};
        a.src = static_cast<const char *>(src); a.src_chunk = (long long)src_chunk_bytes;
        a.src_row = (long long)src_row_bytes;
        a.dst = static_cast<char *>(dst); a.dst_row = (long long)dst_row_bytes;
        a.row_bytes = (long long)row_bytes;
        a.n = std::min(kStitchMaxChunks, n_chunks - c0);
        for (int i = 0; i < a.n; ++i) {
            const vtx_enc_chunk &ch = chunks[c0 + i];
            a.first[i + 1] = a.first[i] + ch.stride;
            a.skip[i] = ch.skip; a.write[i] = ch.write_offset; a.chunk[i] = c0 + i;
        }
        if (a.first[a.n] == 0) continue;
        const dim3 grid((unsigned)std::min(a.first[a.n], ds->sms * 8));
        int r = VTX_OK;
        if (vec == 16) r = launch_pdl(enc_stitch_kernel<16>, grid, dim3(256), 0, st, a);
        else if (vec == 8) r = launch_pdl(enc_stitch_kernel<8>, grid, dim3(256), 0, st, a);
        else if (vec == 4) r = launch_pdl(enc_stitch_kernel<4>, grid, dim3(256), 0, st, a);
        else r = launch_pdl(enc_stitch_kernel<1>, grid, dim3(256), 0, st, a);
        if (r != VTX_OK) return VTX_ERR_CUDA;
    }
    return VTX_OK;
}

int vtx_attn_out_proj(const vtx_out_proj_args *p, void *stream) {
    if (!p || !p->attn || !p->w || !p->dst) return VTX_ERR_NULL;
    const vtx_tensor &A = *p->attn, &W = *p->w, &Y = *p->dst;
    if ((A.type != VTX_TYPE_F32 && A.type != VTX_TYPE_F16) || W.type != VTX_TYPE_F16 || Y.type != VTX_TYPE_F32)
        return VTX_ERR_TYPE;
    const bool af16 = A.type == VTX_TYPE_F16;
    const size_t aes = af16 ? 2 : 4;
    const int64_t Dv = A.ne[0], Hq = A.ne[1], n = A.ne[2];
    if (A.ne[3] != 1 || Dv <= 0 || Dv % 64 || Hq <= 0 || n < 0) return VTX_ERR_SHAPE;
    const int64_t K = Dv * Hq, N = W.ne[1];
    if (W.ne[0] != K || W.ne[2] != 1 || W.ne[3] != 1 || N <= 0) return VTX_ERR_SHAPE;
    if (Y.ne[0] != N || Y.ne[1] != n || Y.ne[2] != 1 || Y.ne[3] != 1) return VTX_ERR_SHAPE;
    if (K > INT32_MAX || N > INT32_MAX || n > INT32_MAX) return VTX_ERR_SHAPE;
    if (n == 0) return VTX_OK;
    if (!A.data || !W.data || !Y.data) return VTX_ERR_NULL;
    const int hb = p->head_block > 0 ? p->head_block : (int)Hq;
    if (Hq % hb) return VTX_ERR_SHAPE;
    const int h_out = (int)(Hq / hb);
    if (A.nb[0] != aes || W.nb[0] != 2 || Y.nb[0] != 4) return VTX_ERR_STRIDE;
    const size_t outer = h_out > 1 ? p->block_nb : A.nb[1] * (size_t)hb;
    const uintptr_t al = reinterpret_cast<uintptr_t>(A.data) | reinterpret_cast<uintptr_t>(W.data) |
                         reinterpret_cast<uintptr_t>(Y.data) | (uintptr_t)A.nb[1] | (uintptr_t)A.nb[2] |
                         (uintptr_t)outer | (uintptr_t)W.nb[1] | (uintptr_t)Y.nb[1];
    if (al % 16) return VTX_ERR_STRIDE;
    const float *bias = nullptr;
    if (p->bias) {
        if (p->bias->type != VTX_TYPE_F32 || p->bias->ne[0] != N || p->bias->nb[0] != 4) return VTX_ERR_SHAPE;
        bias = static_cast<const float *>(p->bias->data);
        if (!bias) return VTX_ERR_NULL;
    }
    const char *res = nullptr;
    long long res_nb1 = 0;
    if (p->residual) {
        const vtx_tensor &R = *p->residual;
        if (R.type != VTX_TYPE_F32 || R.ne[0] != N || R.ne[1] != n || R.nb[0] != 4) return VTX_ERR_SHAPE;
        res = static_cast<const char *>(R.data);
        res_nb1 = (long long)R.nb[1];
        if (!res) return VTX_ERR_NULL;
        if ((reinterpret_cast<uintptr_t>(res) | (uintptr_t)res_nb1) % 16) return VTX_ERR_STRIDE;
    }
    DeviceState *ds = nullptr;
    int rc = ensure_device(&ds);
    if (rc != VTX_OK) return rc;
    if (!g_encode) return VTX_ERR_CUDA;
    CUtensorMap ma, mw, my;
    {
        // A: [Dv, heads in a block, tokens, blocks], one box = 64 columns of one head x 128 tokens
        cuuint64_t dims[4] = {(cuuint64_t)Dv, (cuuint64_t)hb, (cuuint64_t)n, (cuuint64_t)h_out};
        cuuint64_t strides[3] = {(cuuint64_t)(hb > 1 ? A.nb[1] : Dv * aes), (cuuint64_t)(n > 1 ? A.nb[2] : 16),
                                 (cuuint64_t)outer};
        for (int i = 0; i < 3; ++i)
            if (strides[i] == 0 || strides[i] % 16 || strides[i] >= (1ULL << 40)) return VTX_ERR_STRIDE;
        cuuint32_t box[4] = {64, 1, 128, 1}, estr[4] = {1, 1, 1, 1};
        // F16 A lands in the MMA's 128-byte swizzle directly; F32 A unswizzled for the conversion
        if (g_encode(&ma, af16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, A.data, dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     af16 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return VTX_ERR_STRIDE;
    }
    {
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
        cuuint64_t strides[1] = {(cuuint64_t)W.nb[1]};
        cuuint32_t box[2] = {64, 128}, estr[2] = {1, 1};
        if (g_encode(&mw, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, W.data, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return VTX_ERR_STRIDE;
    }
    // the output and the residual: F32 [N, n], boxes of 32 columns x 128 tokens, 128-byte swizzle
    auto rows_map = [&](CUtensorMap *m, void *ptr, size_t nb1) {
        cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)n};
        cuuint64_t strides[1] = {(cuuint64_t)(n > 1 ? nb1 : (size_t)((N * 4 + 15) / 16 * 16))};
        cuuint32_t box[2] = {32, 128}, estr[2] = {1, 1};
        return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, ptr, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    };
    CUtensorMap mr;
    std::memset(&mr, 0, sizeof(mr));
    if (!rows_map(&my, Y.data, Y.nb[1])) return VTX_ERR_STRIDE;
    if (res && !rows_map(&mr, const_cast<char *>(res), (size_t)res_nb1)) return VTX_ERR_STRIDE;
    static std::atomic<int> attr_done[kMaxDevices];
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_done[dev].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(out_proj_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 OutProjCfgT<false>::SMEM) != cudaSuccess ||
            cudaFuncSetAttribute(out_proj_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 OutProjCfgT<true>::SMEM) != cudaSuccess)
            return VTX_ERR_CUDA;
        attr_done[dev].store(1, std::memory_order_release);
    }
    OutProjArgs a{};
    a.M = (int)n; a.N = (int)N; a.K = (int)K; a.Dv = (int)Dv; a.h_in = hb;
    a.bias = bias; a.res = res; a.res_nb1 = res_nb1; a.err = ds->err;
    const dim3 grid((unsigned)((n + OutProjCfg::BM - 1) / OutProjCfg::BM), (unsigned)((N + OutProjCfg::BN - 1) / OutProjCfg::BN));
    if (grid.y > 65535) return VTX_ERR_UNSUPPORTED;
    return af16 ? launch_pdl(out_proj_kernel<true>, grid, dim3(OutProjCfgT<true>::NTHREADS), OutProjCfgT<true>::SMEM,
                             static_cast<cudaStream_t>(stream), ma, mw, my, mr, a)
                : launch_pdl(out_proj_kernel<false>, grid, dim3(OutProjCfg::NTHREADS), OutProjCfg::SMEM,
                             static_cast<cudaStream_t>(stream), ma, mw, my, mr, a);
}

int vtx_read_device_error(void *stream) {
    DeviceState *ds = nullptr;
    int rc = ensure_device(&ds);
    if (rc != VTX_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int h = 0;
    if (cudaMemcpyFromSymbolAsync(&h, g_vtx_kernel_err, sizeof(int), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return VTX_ERR_CUDA;
    if (cudaStreamSynchronize(st) != cudaSuccess) return VTX_ERR_CUDA;
    const int zero = 0;
    if (cudaMemcpyToSymbolAsync(g_vtx_kernel_err, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return VTX_ERR_CUDA;
    if (cudaStreamSynchronize(st) != cudaSuccess) return VTX_ERR_CUDA;
    return h;
}

}  // extern "C"

// ================================================================================
// No-alloc batched decode.
//
// For callers that cannot allocate device memory at all (a plugin inside a
// host application that owns every device allocation, a process under a hard
// memory budget or a custom allocator, a real-time loop that must not block
// in cudaMalloc).  The split-KV partials live in this file-scope buffer
// instead of a caller workspace.  Its host-side name is only a stand-in for
// the device object, so the device address is looked up once per device with
// cudaGetSymbolAddress while that device is current, and that pointer is what
// the kernels receive.  The buffer needs no clearing between calls: every
// partial the combine kernel reads is written earlier in the same call.
// Calls on one device share the buffer, so calls that overlap on the GPU race.
// ================================================================================
static __device__ __align__(256) unsigned char g_vtx_noalloc_scratch[VTX_NOALLOC_SCRATCH_BYTES];

namespace {
std::atomic<void *> g_noalloc_ptr[kMaxDevices];
std::mutex g_noalloc_mu;

// Device address of g_vtx_noalloc_scratch on the current device, looked up
// once per device while that device is current (acquire/release, so a second
// host thread sees either null or the complete address).
int noalloc_scratch(void **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return VTX_ERR_NO_DEVICE;
    void *p = g_noalloc_ptr[dev].load(std::memory_order_acquire);
    if (!p) {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        p = g_noalloc_ptr[dev].load(std::memory_order_relaxed);
        if (!p) {
            if (cudaGetSymbolAddress(&p, g_vtx_noalloc_scratch) != cudaSuccess || !p) {
                cudaGetLastError();
                return VTX_ERR_CUDA;
            }
            g_noalloc_ptr[dev].store(p, std::memory_order_release);
        }
    }
    *out = p;
    return VTX_OK;
}
}  // namespace

extern "C" int vtx_flash_attn_decode_batched_noalloc(const vtx_decode_batch *b, void *stream) {
    return decode_batched_impl(b, nullptr, (size_t)VTX_NOALLOC_SCRATCH_BYTES, static_cast<cudaStream_t>(stream),
                               VTX_ERR_SCRATCH_LIMIT, noalloc_scratch);
}
