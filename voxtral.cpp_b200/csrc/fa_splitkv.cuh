// fa_splitkv.cuh — split-KV flash attention on CUDA cores for sm_100a.
//
// Serves the decode node of src/voxtral.cpp:1802 (n_tokens = 1, mask = NULL,
// the per-token step of run_decoder_step :2438 / run_offline_step :2506),
// ragged multi-stream decode, and every operand combination the tensor-core
// prefill kernel does not take (F32 or Q8_0 K/V with few query rows, odd
// strides).  Memory-bound by design: each CTA streams one KV head's keys for
// one key range ("split") through a cp.async ring of shared-memory stages and
// reuses every K/V row for all query rows of the GQA group (Hq/Hkv heads x
// up to a few tokens), so KV bytes are read from HBM exactly once per split.
//
// Numerics follow ggml's CPU flash_attn_ext (ggml-cpu/ops.cpp @5cecdad):
//   F16 K : dot of half K with Q, fp32 accumulate
//   Q8_0 K: Q quantized per 32-block (d = amax/127, q = rint(x*127/amax)),
//           int8 dot (dp4a) times d_k*d_q per block — ggml's vec_dot_q8_0_q8_0
//   F32 K : fp32 dot
// The softmax runs in the log2 domain (scores pre-multiplied by log2 e),
// V accumulates in fp32.  Partial (m, l, o) per split are merged by
// fa_combine_kernel.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>
#include "vtx_ptx.cuh"

namespace vtx {

struct SplitArgs {
    const char *q; int q_f16; long long q_nb1, q_nb2, q_nb3;
    const char *k, *v; long long k_nb1, k_nb2, k_nb3, v_nb1, v_nb2, v_nb3;
    int k_bdiv, v_bdiv;                       // batch broadcast: ik3 = b / k_bdiv
    const void *const *k_ptrs; const void *const *v_ptrs; const int *kv_len;  // batched mode
    int n_kv;
    const char *mask; long long m_nb1, m_nb2, m_nb3; int m_ne2, m_ne3;
    char *dst; long long d_nb1, d_nb2, d_nb3;  // head, token, batch strides (bytes)
    float *part_o; float *part_ml;
    int n_q, Hq, Hkv, G, B;
    int tok_per_cta, hc, n_hchunks, n_qtiles;
    int chunk, n_splits;
    float qk_scale, softcap, max_bias, m0, m1; int n_head_log2;
    int causal, window;
    int write_final;
    int vec;                                   // cp.async width: 16, 8 or 4 bytes
    int *err;                                  // device error word (misaligned stream base)
    // batched decode: per stream the row written by the kernel just before
    // (-1: none); when set the streaming decode kernels read every other row
    // before waiting for that kernel (programmatic dependent launch)
    const int *fresh;
};

template <int KVT> struct KvTraits;
template <> struct KvTraits<1> { static constexpr int TK = 64; template <int D> static constexpr int row_bytes() { return D * 2; } };
template <> struct KvTraits<0> { static constexpr int TK = 32; template <int D> static constexpr int row_bytes() { return D * 4; } };
template <> struct KvTraits<8> { static constexpr int TK = 64; template <int D> static constexpr int row_bytes() { return D / 32 * 34; } };

template <int D, int KVT> struct SplitCfg {
    static constexpr int TK = KvTraits<KVT>::TK;
    static constexpr int ROW = KvTraits<KVT>::template row_bytes<D>();
    static constexpr int PITCH = ((ROW + 15) / 16) * 16 + 16;     // +16 B: conflict-free row access
    static constexpr int STAGE_BYTES = 2 * TK * PITCH;
    static constexpr int STAGES = KVT == 0 ? 2 : 3;
    static constexpr int NTHREADS = 128;
};

__device__ __forceinline__ float alibi_slope(const SplitArgs &a, int h) {
    if (!(a.max_bias > 0.0f)) return 1.0f;
    return h < a.n_head_log2 ? powf(a.m0, (float)(h + 1)) : powf(a.m1, (float)(2 * (h - a.n_head_log2) + 1));
}

__device__ __forceinline__ void cp_async(void *dst, const void *src, int bytes) {
    const uint32_t d = smem_u32(dst);
    if (bytes == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
    else if (bytes == 8)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(d), "l"(src) : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// 4 bytes starting at a 2-byte aligned shared address.
__device__ __forceinline__ uint32_t lds_u32_unaligned(const char *p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    const uint32_t sh = (uint32_t)(a & 3) * 8;
    return sh ? __funnelshift_r(w[0], w[1], sh) : w[0];
}

__device__ __forceinline__ void h8_to_f(const uint4 &raw, float (&f)[8]) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 t = __half22float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

template <int D, int KVT, int MAXR>
__global__ void __launch_bounds__(128)
fa_splitkv_kernel(const SplitArgs a)
{
    grid_dep_wait();
    grid_dep_launch();
    using C = SplitCfg<D, KVT>;
    constexpr int TK = C::TK, PITCH = C::PITCH, STAGES = C::STAGES;
    constexpr int QP = D / 2 + 4;            // padded half-row of Q (floats)
    extern __shared__ __align__(128) char smem[];
    char *stage_base = smem;
    float *qs = reinterpret_cast<float *>(smem + STAGES * C::STAGE_BYTES);   // [MAXR][2][QP]
    float *ss = qs + MAXR * 2 * QP;                                            // [MAXR][TK]
    float *row_m = ss + MAXR * TK;                                             // [MAXR]
    float *row_l = row_m + MAXR;
    float *row_a = row_l + MAXR;
    float *row_slope = row_a + MAXR;
    int *row_lo = reinterpret_cast<int *>(row_slope + MAXR);
    int *row_hi = row_lo + MAXR;
    int8_t *qq = reinterpret_cast<int8_t *>(row_hi + MAXR);                    // [MAXR][D] (Q8_0 K)
    float *qd = reinterpret_cast<float *>(qq + MAXR * D);                      // [MAXR][D/32]

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int split = blockIdx.x % a.n_splits;
    const int qt = blockIdx.x / a.n_splits;
    const int hchunk = blockIdx.y % a.n_hchunks;
    const int g = blockIdx.y / a.n_hchunks;
    const int b = blockIdx.z;
    const int rows = a.tok_per_cta * a.hc;

    int kv_len = a.n_kv;
    const char *kbase, *vbase;
    if (a.k_ptrs) {
        kv_len = a.kv_len[b];
        if (split * a.chunk >= kv_len && split > 0) return;   // combine reads ceil(kv_len/chunk) splits
        kbase = static_cast<const char *>(a.k_ptrs[b]);
        vbase = static_cast<const char *>(a.v_ptrs[b]);
    } else {
        kbase = a.k + (long long)(b / a.k_bdiv) * a.k_nb3;
        vbase = a.v + (long long)(b / a.v_bdiv) * a.v_nb3;
    }
    kbase += (long long)g * a.k_nb2;
    vbase += (long long)g * a.v_nb2;
    // Per-stream bases are only known here: a base the cp.async width does not
    // divide is reported through the error word and the stream yields zeros.
    const bool misaligned = ((reinterpret_cast<uintptr_t>(kbase) | reinterpret_cast<uintptr_t>(vbase)) % a.vec) != 0;
    if (misaligned && tid == 0 && a.err) atomicCAS(a.err, 0, 7);
    const int off = kv_len - a.n_q;

    // ---- per-row setup ---------------------------------------------------
    if (tid < MAXR) {
        const int r = tid;
        const int tok = qt * a.tok_per_cta + r / a.hc;
        const int h = g * a.G + hchunk * a.hc + r % a.hc;
        int lo = 0, hi = kv_len - 1;
        if (r >= rows || tok >= a.n_q) { lo = 1; hi = 0; }
        else if (a.causal) {
            hi = min(hi, tok + off);
            if (a.window > 0) lo = max(0, tok + off - (a.window - 1));
        }
        row_lo[r] = lo;
        row_hi[r] = hi;
        row_m[r] = -INFINITY;
        row_l[r] = 0.0f;
        row_slope[r] = (r < rows) ? alibi_slope(a, h) : 1.0f;
    }
    // ---- Q rows -> shared (f32, split in halves with padding) ------------
    for (int i = tid; i < MAXR * D; i += blockDim.x) {
        const int r = i / D, d = i % D;
        const int tok = qt * a.tok_per_cta + r / a.hc;
        const int h = g * a.G + hchunk * a.hc + r % a.hc;
        float x = 0.0f;
        if (r < rows && tok < a.n_q) {
            const char *p = a.q + (long long)tok * a.q_nb1 + (long long)h * a.q_nb2 + (long long)b * a.q_nb3;
            x = a.q_f16 ? __half2float(reinterpret_cast<const __half *>(p)[d]) : reinterpret_cast<const float *>(p)[d];
        }
        if (KVT == 1) x = __half2float(__float2half_rn(x));       // ggml: Q -> K's vec_dot type (F16)
        qs[(r * 2 + d / (D / 2)) * QP + d % (D / 2)] = x;
    }
    __syncthreads();
    if (KVT == 8) {   // ggml: Q -> Q8_0 (x86 from_float: d = amax/127, q = rne(x * 127/amax))
        for (int blk = warp; blk < MAXR * (D / 32); blk += 4) {
            const int r = blk / (D / 32), c = blk % (D / 32);
            const int d = c * 32 + lane;
            const float x = qs[(r * 2 + d / (D / 2)) * QP + d % (D / 2)];
            float amax = fabsf(x);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            const float dd = amax / 127.0f;
            const float id = amax != 0.0f ? 127.0f / amax : 0.0f;
            qq[r * D + d] = (int8_t)__float2int_rn(x * id);
            if (lane == 0) qd[r * (D / 32) + c] = __half2float(__float2half_rn(dd));
        }
    }

    // ---- key range of this split ------------------------------------------
    int klo = kv_len, khi = -1;
    for (int r = 0; r < rows; ++r) {
        if (row_lo[r] <= row_hi[r]) { klo = min(klo, row_lo[r]); khi = max(khi, row_hi[r]); }
    }
    const int kb = max(split * a.chunk, klo);
    const int ke = min(min((split + 1) * a.chunk, kv_len), khi + 1);
    const int ntiles = (ke > kb && !misaligned) ? (ke - kb + TK - 1) / TK : 0;

    // ---- async tile loader --------------------------------------------------
    const int vec = a.vec;
    auto load_tile = [&](int t) {
        if (t < ntiles) {
            char *ks = stage_base + (t % STAGES) * C::STAGE_BYTES;
            char *vs = ks + TK * PITCH;
            const int k0 = kb + t * TK;
            const int n = min(TK, ke - k0);
            const int per_row = C::ROW / vec;
            for (int i = tid; i < n * per_row; i += C::NTHREADS) {
                const int rr = i / per_row, cc = (i % per_row) * vec;
                cp_async(ks + rr * PITCH + cc, kbase + (long long)(k0 + rr) * a.k_nb1 + cc, vec);
                cp_async(vs + rr * PITCH + cc, vbase + (long long)(k0 + rr) * a.v_nb1 + cc, vec);
            }
        }
        cp_async_commit();
    };
#pragma unroll
    for (int t = 0; t < STAGES - 1; ++t) load_tile(t);

    constexpr int DPT = 4;                   // output dims per thread in PV
    constexpr int NDC = D / DPT;             // threads across D
    constexpr int NG = C::NTHREADS / NDC;    // key groups
    const int dc = tid % NDC, kg = tid / NDC;
    float acc[MAXR][DPT];
#pragma unroll
    for (int r = 0; r < MAXR; ++r)
#pragma unroll
        for (int j = 0; j < DPT; ++j) acc[r][j] = 0.0f;

    const bool has_mask = a.mask != nullptr;
    for (int t = 0; t < ntiles; ++t) {
        cp_async_wait<STAGES - 2>();
        __syncthreads();
        load_tile(t + STAGES - 1);
        const char *ks = stage_base + (t % STAGES) * C::STAGE_BYTES;
        const char *vs = ks + TK * PITCH;
        const int k0 = kb + t * TK;
        const int n = min(TK, ke - k0);

        // ---- S = Q K^T for this tile ----------------------------------------
        {
            constexpr int KPT = C::NTHREADS / TK;      // threads per key (2 or 4)
            const int kk = tid / KPT, part = tid % KPT;
            constexpr int DP = D / KPT;                // dims per thread
            float sacc[MAXR];
#pragma unroll
            for (int r = 0; r < MAXR; ++r) sacc[r] = 0.0f;
            const char *krow = ks + kk * PITCH;
            if (KVT == 1) {
#pragma unroll
                for (int c = 0; c < DP / 8; ++c) {
                    const int d0 = part * DP + c * 8;
                    float kf[8];
                    h8_to_f(*reinterpret_cast<const uint4 *>(krow + d0 * 2), kf);
#pragma unroll
                    for (int r = 0; r < MAXR; ++r) {
                        const float *qr = qs + (r * 2 + d0 / (D / 2)) * QP + d0 % (D / 2);
                        const float4 q0 = *reinterpret_cast<const float4 *>(qr);
                        const float4 q1 = *reinterpret_cast<const float4 *>(qr + 4);
                        float s = sacc[r];
                        s = fmaf(q0.x, kf[0], s); s = fmaf(q0.y, kf[1], s);
                        s = fmaf(q0.z, kf[2], s); s = fmaf(q0.w, kf[3], s);
                        s = fmaf(q1.x, kf[4], s); s = fmaf(q1.y, kf[5], s);
                        s = fmaf(q1.z, kf[6], s); s = fmaf(q1.w, kf[7], s);
                        sacc[r] = s;
                    }
                }
            } else if (KVT == 0) {
#pragma unroll 4
                for (int c = 0; c < DP / 4; ++c) {
                    const int d0 = part * DP + c * 4;
                    const float4 kf = *reinterpret_cast<const float4 *>(krow + d0 * 4);
#pragma unroll
                    for (int r = 0; r < MAXR; ++r) {
                        const float4 q0 = *reinterpret_cast<const float4 *>(qs + (r * 2 + d0 / (D / 2)) * QP + d0 % (D / 2));
                        float s = sacc[r];
                        s = fmaf(q0.x, kf.x, s); s = fmaf(q0.y, kf.y, s);
                        s = fmaf(q0.z, kf.z, s); s = fmaf(q0.w, kf.w, s);
                        sacc[r] = s;
                    }
                }
            } else {   // Q8_0
#pragma unroll
                for (int c = 0; c < DP / 32; ++c) {
                    const int blk = (part * DP) / 32 + c;
                    const char *bp = krow + blk * 34;
                    const float dk = __half2float(*reinterpret_cast<const __half *>(bp));
                    uint32_t kw[8];
#pragma unroll
                    for (int w = 0; w < 8; ++w) kw[w] = lds_u32_unaligned(bp + 2 + 4 * w);
#pragma unroll
                    for (int r = 0; r < MAXR; ++r) {
                        const int *qw = reinterpret_cast<const int *>(qq + r * D + blk * 32);
                        int isum = 0;
#pragma unroll
                        for (int w = 0; w < 8; ++w) isum = __dp4a((int)kw[w], qw[w], isum);
                        sacc[r] = fmaf(dk * qd[r * (D / 32) + blk], (float)isum, sacc[r]);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < MAXR; ++r) {
#pragma unroll
                for (int o = 1; o < KPT; o <<= 1) sacc[r] += __shfl_xor_sync(0xffffffffu, sacc[r], o);
            }
            if (part == 0) {
                const int j = k0 + kk;
#pragma unroll
                for (int r = 0; r < MAXR; ++r) {
                    if (r < rows) {
                        float s = -INFINITY;
                        if (kk < n && j >= row_lo[r] && j <= row_hi[r]) {
                            s = sacc[r] * a.qk_scale;
                            if (a.softcap != 0.0f) s = a.softcap * tanhf(s);
                            if (has_mask) {
                                const int tok = qt * a.tok_per_cta + r / a.hc;
                                const int h = g * a.G + hchunk * a.hc + r % a.hc;
                                const char *mp = a.mask + (long long)tok * a.m_nb1 + (long long)(h % a.m_ne2) * a.m_nb2 +
                                                 (long long)(b % a.m_ne3) * a.m_nb3;
                                const float mv = row_slope[r] * __half2float(reinterpret_cast<const __half *>(mp)[j]);
                                s = (mv == -INFINITY) ? -INFINITY : s + mv;
                            }
                            s *= kLog2e;
                        }
                        ss[r * TK + kk] = s;
                    }
                }
            }
        }
        __syncthreads();

        // ---- online softmax, one warp per row ---------------------------------
        for (int r = warp; r < rows; r += 4) {
            float mx = -INFINITY;
            for (int kk = lane; kk < TK; kk += 32) mx = fmaxf(mx, ss[r * TK + kk]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float m_old = row_m[r];
            const float m_new = fmaxf(m_old, mx);
            const float m_use = m_new == -INFINITY ? 0.0f : m_new;
            float sum = 0.0f;
            for (int kk = lane; kk < TK; kk += 32) {
                const float p = ex2(ss[r * TK + kk] - m_use);
                ss[r * TK + kk] = p;
                sum += p;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            if (lane == 0) {
                const float alpha = ex2(m_old - m_use);       // m_old = -inf -> 0 (acc is 0 anyway)
                row_a[r] = alpha;
                row_l[r] = row_l[r] * alpha + sum;
                row_m[r] = m_new;
            }
        }
        __syncthreads();

        // ---- O += P V ----------------------------------------------------------
#pragma unroll
        for (int r = 0; r < MAXR; ++r) {
            const float al = r < rows ? row_a[r] : 1.0f;
#pragma unroll
            for (int j = 0; j < DPT; ++j) acc[r][j] *= al;
        }
        for (int kk = kg; kk < n; kk += NG) {
            float vf[4];
            const char *vrow = vs + kk * PITCH;
            if (KVT == 1) {
                const uint2 raw = *reinterpret_cast<const uint2 *>(vrow + dc * DPT * 2);
                const float2 v01 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
                const float2 v23 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
                vf[0] = v01.x; vf[1] = v01.y; vf[2] = v23.x; vf[3] = v23.y;
            } else if (KVT == 0) {
                const float4 t4 = *reinterpret_cast<const float4 *>(vrow + dc * DPT * 4);
                vf[0] = t4.x; vf[1] = t4.y; vf[2] = t4.z; vf[3] = t4.w;
            } else {
                const int d0 = dc * DPT;
                const char *bp = vrow + (d0 / 32) * 34;
                const float dv = __half2float(*reinterpret_cast<const __half *>(bp));
                const uint32_t w = lds_u32_unaligned(bp + 2 + (d0 % 32));
#pragma unroll
                for (int j = 0; j < 4; ++j) vf[j] = dv * (float)(int8_t)((w >> (8 * j)) & 0xff);
            }
#pragma unroll
            for (int r = 0; r < MAXR; ++r) {
                const float p = ss[r * TK + kk];
#pragma unroll
                for (int j = 0; j < DPT; ++j) acc[r][j] = fmaf(p, vf[j], acc[r][j]);
            }
        }
    }
    cp_async_wait<0>();
    __syncthreads();

    // ---- reduce the NG key groups and write ---------------------------------
    float *red = reinterpret_cast<float *>(stage_base);        // [NG][MAXR][D]
#pragma unroll
    for (int r = 0; r < MAXR; ++r)
#pragma unroll
        for (int j = 0; j < DPT; ++j) red[(kg * MAXR + r) * D + dc * DPT + j] = acc[r][j];
    __syncthreads();
    const long long work = (((long long)b * gridDim.y + blockIdx.y) * a.n_qtiles + qt) * a.n_splits + split;
    for (int i = tid; i < rows * D; i += C::NTHREADS) {
        const int r = i / D, d = i % D;
        float o = 0.0f;
#pragma unroll
        for (int q = 0; q < NG; ++q) o += red[(q * MAXR + r) * D + d];
        const int tok = qt * a.tok_per_cta + r / a.hc;
        if (tok >= a.n_q) continue;
        if (a.write_final) {
            const int h = g * a.G + hchunk * a.hc + r % a.hc;
            const float l = row_l[r];
            float *out = reinterpret_cast<float *>(a.dst + (long long)tok * a.d_nb2 + (long long)h * a.d_nb1 +
                                                   (long long)b * a.d_nb3);
            out[d] = l == 0.0f ? 0.0f : o / l;
        } else {
            a.part_o[(work * MAXR + r) * D + d] = o;
            if (d == 0) {
                a.part_ml[(work * MAXR + r) * 2 + 0] = row_m[r];
                a.part_ml[(work * MAXR + r) * 2 + 1] = row_l[r];
            }
        }
    }
}

// Merge split partials: one CTA of NT threads per output row, so that at
// batch 1 (a few dozen rows, up to hundreds of splits) the loads of all splits
// are in flight together instead of one split after another.
//   1. M = max over the splits' maxima (block reduction);
//   2. thread (split group sg, float4 column c) sums f_s * o_s[c] over the
//      splits s = sg, sg + NSG, ... with f_s = 2^(m_s - M) (0 for an empty
//      split), and the block sums l_s * f_s;
//   3. the NSG column partials are added in shared memory and scaled by 1/L.
template <int D, int MAXR, int NT>
__global__ void __launch_bounds__(NT)
fa_combine_kernel(const SplitArgs a, int gy)
{
    grid_dep_wait();
    grid_dep_launch();
    constexpr int C4 = D / 4, NSG = NT / C4;                   // float4 columns, split groups
    __shared__ float4 acc_s[NSG][C4];
    const int tid = threadIdx.x;
    const long long row_id = blockIdx.x;
    const int rows = a.tok_per_cta * a.hc;
    const int r = (int)(row_id % rows);
    long long t = row_id / rows;
    const int qt = (int)(t % a.n_qtiles); t /= a.n_qtiles;
    const int y = (int)(t % gy);
    const int b = (int)(t / gy);
    if (b >= a.B) return;
    const int hchunk = y % a.n_hchunks, g = y / a.n_hchunks;
    const int tok = qt * a.tok_per_cta + r / a.hc;
    if (tok >= a.n_q) return;                                  // uniform over the CTA
    const int h = g * a.G + hchunk * a.hc + r % a.hc;
    int nsp = a.n_splits;
    if (a.k_ptrs) nsp = max(1, min(a.n_splits, (a.kv_len[b] + a.chunk - 1) / a.chunk));
    const long long w0 = (((long long)b * gy + y) * a.n_qtiles + qt) * a.n_splits;
    const float *ml = a.part_ml + (w0 * MAXR + r) * 2;             // split s at ml[s * MAXR * 2]
    const float *po0 = a.part_o + (w0 * MAXR + r) * D;             // split s at po0[s * MAXR * D]

    // One load round: thread (split group sg, float4 column c) merges the
    // splits sg, sg + NSG, ... online (its own running max, four splits'
    // loads in flight), then the groups are merged in shared memory in group
    // order -- the same order on every run.
    __shared__ float grp_m[NSG], grp_l[NSG];
    const int c = tid % C4, sg = tid / C4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float m_t = -INFINITY, l_t = 0.0f;
    auto fold = [&](float m, float l, const float4 &x) {
        if (l == 0.0f) return;                                 // a split with no key (or an empty row)
        if (m > m_t) {
            const float f = m_t == -INFINITY ? 0.0f : ex2(m_t - m);
            acc.x *= f; acc.y *= f; acc.z *= f; acc.w *= f;
            l_t *= f;
            m_t = m;
        }
        const float w = ex2(m - m_t);
        acc.x = fmaf(w, x.x, acc.x); acc.y = fmaf(w, x.y, acc.y);
        acc.z = fmaf(w, x.z, acc.z); acc.w = fmaf(w, x.w, acc.w);
        l_t = fmaf(w, l, l_t);
    };
    int s = sg;
    for (; s + 3 * NSG < nsp; s += 4 * NSG) {
        float2 mlu[4];
        float4 x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const long long su = s + u * NSG;
            mlu[u] = *reinterpret_cast<const float2 *>(ml + su * MAXR * 2);
            x[u] = reinterpret_cast<const float4 *>(po0 + su * MAXR * D)[c];
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) fold(mlu[u].x, mlu[u].y, x[u]);
    }
    for (; s < nsp; s += NSG) {
        const float2 m2 = *reinterpret_cast<const float2 *>(ml + (long long)s * MAXR * 2);
        fold(m2.x, m2.y, reinterpret_cast<const float4 *>(po0 + (long long)s * MAXR * D)[c]);
    }
    acc_s[sg][c] = acc;
    if (c == 0) {
        grp_m[sg] = m_t;
        grp_l[sg] = l_t;
    }
    __syncthreads();
    if (tid < C4) {
        float M = -INFINITY;
#pragma unroll
        for (int q = 0; q < NSG; ++q) M = fmaxf(M, grp_m[q]);
        float L = 0.0f;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int q = 0; q < NSG; ++q) {
            if (grp_l[q] == 0.0f) continue;
            const float w = ex2(grp_m[q] - M);
            const float4 v = acc_s[q][tid];
            o.x = fmaf(w, v.x, o.x); o.y = fmaf(w, v.y, o.y);
            o.z = fmaf(w, v.z, o.z); o.w = fmaf(w, v.w, o.w);
            L = fmaf(w, grp_l[q], L);
        }
        const float inv = L == 0.0f ? 0.0f : 1.0f / L;
        float *out = reinterpret_cast<float *>(a.dst + (long long)tok * a.d_nb2 + (long long)h * a.d_nb1 +
                                               (long long)b * a.d_nb3);
        out[4 * tid + 0] = o.x * inv; out[4 * tid + 1] = o.y * inv;
        out[4 * tid + 2] = o.z * inv; out[4 * tid + 3] = o.w * inv;
    }
}

template <int D, int KVT, int MAXR>
constexpr int splitkv_smem_bytes() {
    using C = SplitCfg<D, KVT>;
    int s = C::STAGES * C::STAGE_BYTES;
    const int red = (C::NTHREADS / (D / 4)) * MAXR * D * 4;
    if (red > s) s = red;
    s += MAXR * 2 * (D / 2 + 4) * 4 + MAXR * C::TK * 4 + MAXR * 6 * 4 + MAXR * D + MAXR * (D / 32) * 4;
    return (s + 15) / 16 * 16;
}

}  // namespace vtx
