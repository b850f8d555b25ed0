// fa_decode_q8.cuh — HBM-streaming decode attention over a Q8_0 KV cache
// (sm_100a).
//
// The decode node of src/voxtral.cpp:1802 with the cache quantised to Q8_0
// (ggml blocks {f16 d; int8 qs[32]}, 34 bytes per 32 values): one decode token
// per stream reads every cache byte once, so the kernel is bound by HBM.
// A head's row is 136 bytes (D = 128) and only 8-byte aligned, so per-head
// rows cannot be bulk-copied.  Instead one CTA covers HPC consecutive KV heads
// (all 8 of voxtral's decoder) of one (stream, key split):
//
//   warp HPC_MAX    producer: lane l bulk-copies the HPC-head slice of token
//                   row l (K, l < 16) or l - 16 (V) of a 16-key stage into a
//                   3-stage ring — HPC * 136 bytes, contiguous and 16-byte
//                   aligned; completion counted by one mbarrier per stage,
//                   reuse gated by a second one (one arrival per head warp).
//   warp w < HPC    head h0 + w: dequantises its K slices of the stage into
//                   a private f16 tile (two lanes per key, 68 bytes = two
//                   blocks each; ring rows are padded by 16 B so the lanes
//                   meet at most 2 to a bank; int8 -> f16 exactly through the
//                   0x64xx bit pattern, then times the block scale, rounded
//                   once to f16), computes S = Q K^T and the softmax on the
//                   tensor core (decode_scores, the F16 kernel's step, G
//                   query heads as the M rows), then dequantises V into the
//                   same tile, releases the ring stage and adds P V.  One
//                   tile per warp leaves room for a 5-stage ring, so ~140 KB
//                   of a CTA's rows are in flight.
//
// Q is quantised to Q8_0 per 32 values first, as ggml's CPU kernel does before
// its Q8_0 dot (d = amax/127, q = round-half-even(x * 127/amax)), and fed to
// the MMA as f16(d * q).  Partials use fa_combine_kernel's layout.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>
#include "vtx_ptx.cuh"
#include "fa_splitkv.cuh"
#include "fa_decode_mma.cuh"

namespace vtx {

template <int D> struct DecodeQ8Cfg {
    static_assert(D == 128, "Q8_0 streaming decode is built for head_dim 128");
    static constexpr int KEYS = 16;                          // keys per stage
    static constexpr int STAGES = 5;                         // ~140 KB of a CTA's rows in flight
    static constexpr int HPC_MAX = 8;                        // KV heads per CTA (= head warps)
    static constexpr int BLK = D / 32 * 34;                  // one head's Q8_0 row (136 B)
    static constexpr int RING_STAGE = 2 * KEYS * (HPC_MAX * BLK + 16);   // rows padded by 16 B
    static constexpr int FPITCH = D * 2 + 16;                // dequantised f16 row pitch
    static constexpr int WBUF = KEYS * FPITCH;               // one head warp's f16 tile (K, then V)
    static constexpr int BUF_OFF = STAGES * RING_STAGE;
    static constexpr int BAR_OFF = BUF_OFF + HPC_MAX * WBUF;
    static constexpr int SMEM = BAR_OFF + 2 * STAGES * 8;
    static constexpr int NTHREADS = (HPC_MAX + 1) * 32;
};

// 4 int8 (one 32-bit word) -> two f16x2, each value d * q rounded to half.
__device__ __forceinline__ void q8x4_to_h2(uint32_t w, __half2 d2, uint32_t &lo, uint32_t &hi) {
    const uint32_t u = w ^ 0x80808080u;                      // q + 128, as unsigned bytes
    uint32_t a, b;
    asm("prmt.b32 %0, %1, %2, 0x5140;" : "=r"(a) : "r"(u), "r"(0x64646464u));   // {0x64, u0}, {0x64, u1}
    asm("prmt.b32 %0, %1, %2, 0x5342;" : "=r"(b) : "r"(u), "r"(0x64646464u));   // {0x64, u2}, {0x64, u3}
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));   // 1152
    __half2 fa = __hsub2(*reinterpret_cast<__half2 *>(&a), bias);    // exact q
    __half2 fb = __hsub2(*reinterpret_cast<__half2 *>(&b), bias);
    fa = __hmul2(fa, d2);                                    // exact product, one rounding
    fb = __hmul2(fb, d2);
    lo = *reinterpret_cast<uint32_t *>(&fa);
    hi = *reinterpret_cast<uint32_t *>(&fb);
}

// Half of one head's Q8_0 row: two blocks (68 bytes from a 4-byte aligned
// shared-memory address) -> 64 halves written to dst (16-byte aligned).
// The first block's int8 values sit at a 2-byte offset (funnel shifts), the
// second block's on word boundaries.
__device__ __forceinline__ void dequant_2blocks(const char *src, char *dst) {
    uint32_t w[17];
#pragma unroll
    for (int i = 0; i < 17; ++i) w[i] = reinterpret_cast<const uint32_t *>(src)[i];
    const __half dA = __ushort_as_half((unsigned short)(w[0] & 0xffffu));   // bytes 0-1
    const __half dB = __ushort_as_half((unsigned short)(w[8] >> 16));       // bytes 34-35
    const __half2 dA2 = __halves2half2(dA, dA), dB2 = __halves2half2(dB, dB);
    uint32_t out[32];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        q8x4_to_h2(__funnelshift_r(w[j], w[j + 1], 16), dA2, out[2 * j], out[2 * j + 1]);   // bytes 2..33
        q8x4_to_h2(w[9 + j], dB2, out[16 + 2 * j], out[16 + 2 * j + 1]);                  // bytes 36..67
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
        reinterpret_cast<uint4 *>(dst)[i] = make_uint4(out[4 * i], out[4 * i + 1], out[4 * i + 2], out[4 * i + 3]);
}

template <int D>
__global__ void __launch_bounds__(DecodeQ8Cfg<D>::NTHREADS, 1)
fa_decode_q8_kernel(const SplitArgs a, int hpc)
{
    grid_dep_wait();
    grid_dep_launch();
    using C = DecodeQ8Cfg<D>;
    constexpr int KC = D / 16, NB = D / 8;
    extern __shared__ __align__(128) char smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *empty = full + C::STAGES;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // work item: (stream b, head group hg, key split sp)
    const int ngroups = a.Hkv / hpc;
    const int hg = blockIdx.x % ngroups;
    const int sp = (blockIdx.x / ngroups) % a.n_splits;
    const int b = blockIdx.x / (ngroups * a.n_splits);
    const int trow = hpc * C::BLK;                           // bytes copied per token row
    const int tpitch = trow + 16;                            // padded ring row: rows rotate banks

    int kv_len = a.n_kv;
    const char *kbase, *vbase;
    if (a.k_ptrs) {
        kv_len = a.kv_len[b];
        kbase = static_cast<const char *>(a.k_ptrs[b]);
        vbase = static_cast<const char *>(a.v_ptrs[b]);
    } else {
        kbase = a.k + (long long)(b / a.k_bdiv) * a.k_nb3;
        vbase = a.v + (long long)(b / a.v_bdiv) * a.v_nb3;
    }
    kbase += (long long)hg * hpc * a.k_nb2;
    vbase += (long long)hg * hpc * a.v_nb2;
    const int kb = sp * a.chunk;
    const int ke = min(kb + a.chunk, kv_len);
    // splits past this stream's length are not read by the combine kernel
    if (a.k_ptrs && sp > 0 && kb >= kv_len) return;
    const bool misaligned = ((reinterpret_cast<uintptr_t>(kbase) | reinterpret_cast<uintptr_t>(vbase) |
                              (uintptr_t)a.k_nb1 | (uintptr_t)a.v_nb1) & 15) != 0;
    if (misaligned && threadIdx.x == 0 && a.err) atomicCAS(a.err, 0, 7);
    const int ntiles = (ke > kb && !misaligned) ? (ke - kb + C::KEYS - 1) / C::KEYS : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], hpc);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == C::HPC_MAX) {
        // ================= producer =========================================
        int issued = 0;
        for (int t = 0; t < ntiles; ++t) {
            const int stg = t % C::STAGES;
            if (t >= C::STAGES &&
                !__all_sync(0xffffffffu, mbar_wait(&empty[stg], ((t / C::STAGES) - 1) & 1, a.err, VTX_KERR_KV)))
                break;
            const int k0 = kb + t * C::KEYS;
            const int n = min(C::KEYS, ke - k0);
            char *st = smem + stg * C::RING_STAGE;
            if (lane == 0) mbar_arrive_expect_tx(&full[stg], (uint32_t)(2 * n * trow));
            __syncwarp();
            const int r = lane & 15;
            if (r < n) {
                if (lane < 16)
                    bulk_g2s(st + r * tpitch, kbase + (long long)(k0 + r) * a.k_nb1, (uint32_t)trow, &full[stg]);
                else
                    bulk_g2s(st + (C::KEYS + r) * tpitch, vbase + (long long)(k0 + r) * a.v_nb1, (uint32_t)trow,
                             &full[stg]);
            }
            issued = t + 1;
        }
        // the CTA's shared memory must outlive every copy still in flight (bounded)
        for (int t = issued > C::STAGES ? issued - C::STAGES : 0; t < issued; ++t)
            mbar_wait(&full[t % C::STAGES], (t / C::STAGES) & 1, nullptr, 0);
        return;
    }
    if (warp >= hpc) return;

    // ==================== head warp ============================================
    const int g = hg * hpc + warp;                           // KV head
    char *buf = smem + C::BUF_OFF + warp * C::WBUF;          // dequantised K, then V, of a stage

    // Q rows of the group as the A fragment (rows >= G are zero), quantised to
    // Q8_0 per 32 values like ggml's from_float for a Q8_0 K
    const int qrow = lane >> 2;
    uint32_t qa[KC][4];
    {
        const bool rq = qrow < a.G;
        const char *qp = a.q + (long long)(g * a.G + (rq ? qrow : 0)) * a.q_nb2 + (long long)b * a.q_nb3;
        float x[KC][4];
#pragma unroll
        for (int kc = 0; kc < KC; ++kc) {
            const int c = kc * 16 + 2 * (lane & 3);
            x[kc][0] = x[kc][1] = x[kc][2] = x[kc][3] = 0.f;
            if (rq) {
                if (a.q_f16) {
                    const __half *hq = reinterpret_cast<const __half *>(qp);
                    x[kc][0] = __half2float(hq[c]); x[kc][1] = __half2float(hq[c + 1]);
                    x[kc][2] = __half2float(hq[c + 8]); x[kc][3] = __half2float(hq[c + 9]);
                } else {
                    const float *fq = reinterpret_cast<const float *>(qp);
                    x[kc][0] = fq[c]; x[kc][1] = fq[c + 1]; x[kc][2] = fq[c + 8]; x[kc][3] = fq[c + 9];
                }
            }
        }
        // a 32-value block = chunks kc = 2j, 2j+1; its values sit in the 4 lanes of the row
#pragma unroll
        for (int j = 0; j < KC / 2; ++j) {
            float amax = 0.f;
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int i = 0; i < 4; ++i) amax = fmaxf(amax, fabsf(x[2 * j + h][i]));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            const float dq = __half2float(__float2half_rn(amax / 127.0f));
            const float id = amax != 0.0f ? 127.0f / amax : 0.0f;
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int i = 0; i < 4; ++i) x[2 * j + h][i] = dq * (float)__float2int_rn(x[2 * j + h][i] * id);
        }
#pragma unroll
        for (int kc = 0; kc < KC; ++kc) {
            qa[kc][0] = pack_half2(x[kc][0], x[kc][1]);
            qa[kc][1] = 0u;
            qa[kc][2] = pack_half2(x[kc][2], x[kc][3]);
            qa[kc][3] = 0u;
        }
    }

    float o[NB][4];
#pragma unroll
    for (int i = 0; i < NB; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m_run = -INFINITY, l_part = 0.f;
    const float cx = a.qk_scale * kLog2e;
    const int kr = lane >> 1, half = lane & 1;               // dequant: key row, which 2 of its 4 blocks
    char *frow = buf + kr * C::FPITCH + half * 128;

    for (int t = 0; t < ntiles; ++t) {
        const int stg = t % C::STAGES;
        if (!__all_sync(0xffffffffu, mbar_wait(&full[stg], (t / C::STAGES) & 1, a.err, VTX_KERR_KV))) break;
        const int k0 = kb + t * C::KEYS;
        const int n = min(C::KEYS, ke - k0);
        const char *st = smem + stg * C::RING_STAGE + warp * C::BLK + half * 68;
        // keys past the range were never loaded: zeros, so P = 0 multiplies zeros
        auto stage_rows = [&](int r0) {
            if (kr < n) {
                dequant_2blocks(st + (r0 + kr) * tpitch, frow);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) reinterpret_cast<uint4 *>(frow)[i] = make_uint4(0u, 0u, 0u, 0u);
            }
            __syncwarp();
        };
        uint32_t pa[4];
        stage_rows(0);                                       // K
        decode_scores<D, C::FPITCH>(buf, n, qa, cx, o, m_run, l_part, lane, pa);
        __syncwarp();                                        // K tile read before it is overwritten
        stage_rows(C::KEYS);                                 // V
        if (lane == 0) mbar_arrive(&empty[stg]);             // this warp is done with the ring stage
        decode_pv<D, C::FPITCH>(buf, pa, o, lane);
        __syncwarp();                                        // V tile read before the next stage's K
    }
    decode_store<D>(a, b, g, sp, o, m_run, l_part, lane);
}

}  // namespace vtx
