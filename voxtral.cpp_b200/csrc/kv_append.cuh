// kv_append.cuh — decoder KV-cache update for sm_100a: RoPE of Q and K and the
// K/V cache write, fused into one HBM-bound pass.
//
// Replaces, per decoder layer, the two ggml_rope_ext nodes, the ggml_cont and
// the two ggml_cpy nodes of src/voxtral.cpp:1744-1770, and the shift-left
// memmove of the cache window (src/voxtral.cpp:1237-1266): each token's rows
// go to a caller-chosen cache row (a ring slot), and decode attention over the
// cache is invariant to the order of its rows.
//
// RoPE follows ggml's mode 0 ("normal": adjacent pairs (x[2i], x[2i+1])) with
// freq_scale 1, ext_factor 0, attn_factor 1, as voxtral.cpp calls it.  Like
// ggml's CPU rope cache, the angle of pair i is the float recurrence
// theta_0 = (float)pos, theta_{i+1} = theta_i * theta_scale with
// theta_scale = powf(freq_base, -2/head_dim) computed on the host, so the
// angles are the same floats ggml uses; cos/sin are taken in double and
// rounded to float (the correctly rounded values).
//
// A CTA per token (many tokens) or per (token, 8 rows) (a few tokens: a
// decode step) builds the token's cos/sin table when it holds a Q or K row;
// each warp streams one row (tensor, head) at a time, a lane owning
// head_dim/32 consecutive elements.
// Cache types: F32 (the reference's own cache), F16 (round to nearest even)
// and Q8_0 (per 32 values d = amax/127 stored as f16,
// q = round-half-even(x * 127/amax), as ggml's CPU from_float; a block is
// 32/E lanes, amax by shuffles).
#pragma once
#include <cuda_fp16.h>
#include <cstdint>
#include "vtx_ptx.cuh"

namespace vtx {

// ggml mode-0 rotation of one adjacent pair by (cos, sin) = c.  Shared by
// every kernel that rotates Q or K, so all of them produce the same floats.
__device__ __forceinline__ void rope_pair(float &x0, float &x1, float2 c) {
    const float a0 = x0, a1 = x1;
    x0 = a0 * c.x - a1 * c.y;
    x1 = a0 * c.y + a1 * c.x;
}

// (cos, sin) of rotation pair i at position pos, as ggml's CPU rope cache:
// theta_0 = (float)pos, theta_{i+1} = theta_i * theta_scale, then sin and cos
// in double rounded to float.
__device__ __forceinline__ float2 rope_cs(float theta) {
    double sd, cd;
    sincos((double)theta, &sd, &cd);
    return make_float2((float)cd, (float)sd);
}

// One lane's E consecutive values of a head row written as Q8_0 into the
// head's cache bytes `row` (blocks of 34 bytes: f16 d, then 32 int8): 32 / E
// lanes share a block, amax by shuffles, d = amax/127 rounded to half,
// q = round-half-even(x * 127/amax) -- ggml's CPU from_float.  Warp-collective.
template <int E>
__device__ __forceinline__ void store_q8_lane(const float (&x)[E], char *row, int lane) {
    constexpr int LPB = 32 / E;
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < E; ++i) amax = fmaxf(amax, fabsf(x[i]));
#pragma unroll
    for (int o = 1; o < LPB; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float id = amax != 0.f ? 127.f / amax : 0.f;
    char *blk = row + (lane / LPB) * 34;
    if (lane % LPB == 0) *reinterpret_cast<__half *>(blk) = __float2half_rn(amax / 127.f);
    // the block's values start 2 bytes in: 2-byte stores stay aligned
    unsigned short *qs = reinterpret_cast<unsigned short *>(blk + 2 + (lane % LPB) * E);
#pragma unroll
    for (int i = 0; i < E; i += 2) {
        const uint32_t q0 = (uint32_t)(__float2int_rn(x[i] * id) & 0xff);
        const uint32_t q1 = (uint32_t)(__float2int_rn(x[i + 1] * id) & 0xff);
        qs[i / 2] = (unsigned short)(q0 | (q1 << 8));
    }
}

struct KvAppendArgs {
    int T, Hq, Hkv, kv_type;
    float theta_scale;
    const float *q; long long q_nb1;        // token stride (floats); heads contiguous
    const float *k; long long k_nb1;
    const float *v; long long v_nb1;
    float *q_out; long long qo_nb1;
    const int *positions, *slots;
    char *k_cache, *v_cache;
    const void *const *k_ptrs; const void *const *v_ptrs;   // optional per-token cache bases
    long long cache_nb1;                    // bytes per cache row
    int rows_per_cta;                       // rows of a token one CTA handles
};

// Grid (tokens, ceil((Hq + 2 Hkv) / rows_per_cta)), 8 warps: threads
// 0..D/2-1 build the token's cos/sin table in shared memory (thread i runs
// the float angle recurrence i steps, then one double-precision sincos
// rounded to float), then the warps take the CTA's rows of the token's
// Hq + 2 Hkv rows, one row per warp at a time.
template <int D>
__global__ void __launch_bounds__(256)
kv_append_kernel(const KvAppendArgs a)
{
    grid_dep_wait();
    grid_dep_launch();
    constexpr int E = D / 32;                               // elements per lane
    __shared__ float2 cs[D / 2];                            // (cos, sin) of pair i
    const int t = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // rows of a token: Q heads, then K heads, then V heads; this CTA takes
    // rows [r0, r0 + rows_per_cta), a warp per row at a time
    const int nwarps = blockDim.x >> 5, r0 = blockIdx.y * a.rows_per_cta;
    const bool rope = r0 < a.Hq + a.Hkv;                     // some Q or K row here
    if (rope && threadIdx.x < D / 2) {
        float theta = (float)a.positions[t];
        for (int i = 0; i < (int)threadIdx.x; ++i) theta *= a.theta_scale;
        cs[threadIdx.x] = rope_cs(theta);
    }
    __syncthreads();
    const int slot = a.slots[t];
    const int per_tok = a.Hq + 2 * a.Hkv;
    for (int r = r0 + warp; r < min(r0 + a.rows_per_cta, per_tok); r += nwarps) {
        const int kind = r < a.Hq ? 0 : (r < a.Hq + a.Hkv ? 1 : 2);   // Q, K, V
        const int h = kind == 0 ? r : (kind == 1 ? r - a.Hq : r - a.Hq - a.Hkv);
        const float *src = kind == 0 ? a.q + (long long)t * a.q_nb1
                                     : (kind == 1 ? a.k + (long long)t * a.k_nb1 : a.v + (long long)t * a.v_nb1);
        src += (long long)h * D + lane * E;
        float x[E];
#pragma unroll
        for (int i = 0; i < E; i += 2) {
            const float2 p = *reinterpret_cast<const float2 *>(src + i);
            x[i] = p.x;
            x[i + 1] = p.y;
        }
        if (kind != 2) {
#pragma unroll
            for (int j = 0; j < E / 2; ++j) rope_pair(x[2 * j], x[2 * j + 1], cs[lane * E / 2 + j]);
        }
        if (kind == 0) {
            float *dst = a.q_out + (long long)t * a.qo_nb1 + (long long)h * D + lane * E;
#pragma unroll
            for (int i = 0; i < E; i += 2) *reinterpret_cast<float2 *>(dst + i) = make_float2(x[i], x[i + 1]);
            continue;
        }
        char *base = kind == 1 ? (a.k_ptrs ? (char *)a.k_ptrs[t] : a.k_cache)
                               : (a.v_ptrs ? (char *)a.v_ptrs[t] : a.v_cache);
        char *crow = base + (long long)slot * a.cache_nb1;
        if (a.kv_type == 0) {                               // F32
            float *dst = reinterpret_cast<float *>(crow) + (long long)h * D + lane * E;
#pragma unroll
            for (int i = 0; i < E; i += 2) *reinterpret_cast<float2 *>(dst + i) = make_float2(x[i], x[i + 1]);
        } else if (a.kv_type == 1) {                        // F16
            __half *dst = reinterpret_cast<__half *>(crow) + (long long)h * D + lane * E;
#pragma unroll
            for (int i = 0; i < E; i += 2)
                *reinterpret_cast<__half2 *>(dst + i) = __floats2half2_rn(x[i], x[i + 1]);
        } else {                                            // Q8_0: 32 / E lanes per block
            store_q8_lane<E>(x, crow + (long long)h * (D / 32) * 34, lane);
        }
    }
}

}  // namespace vtx
