// fa_prefill_sm100.cuh — tensor-core flash attention for sm_100a (tcgen05).
//
// The encoder node (src/voxtral.cpp:1611: 1500 tokens per chunk, head_dim 64,
// bidirectional or causal + 750 window) and the decoder prefill node
// (src/voxtral.cpp:1802: GQA 32/8, head_dim 128, causal) are compute-bound.
// One CTA owns NQT 128-row Q tiles of one KV head (GQA: the G query heads of
// the group are packed into the rows, row = token * G + head-in-group, so
// every K/V tile feeds all of them) and walks the key tiles:
//
//   warp 4*NQT      TMA producer: K_j, V_j (128 keys x D, 128-byte swizzle)
//                   into a STAGES-deep shared-memory ring (mbarrier tx count)
//   warp 4*NQT+1    MMA issuer (one thread): S_t = Q_t K_j^T  (SS, f16->f32,
//                   TMEM), then O_t += P_t V_j with P read from TMEM (TS)
//   warps 0..4*NQT-1  softmax, one warpgroup per Q tile, one thread per row
//                   (= TMEM lane): tcgen05.ld S, scale/mask in the log2
//                   domain, running max with lazy rescaling (only when the
//                   max grows by more than 2^8), P = exp2(S - m) packed to
//                   half into the S columns, O rescaled in TMEM when needed.
//
// TMEM columns: S_t at t*128 (P_t aliases its first 64), O_t after the S
// block.  Causal / windowed key tiles outside every row's range are never
// loaded.  Numerics: Q and P in f16 (Q is rounded to half exactly as ggml
// rounds Q for an F16 K), fp32 accumulation of S and O.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "vtx_ptx.cuh"

namespace vtx {

struct PrefillArgs {
    const char *q; int q_f16; long long q_nb1, q_nb2, q_nb3;
    const char *mask; long long m_nb1, m_nb2, m_nb3; int m_ne2, m_ne3;
    char *dst; long long d_nb1, d_nb2, d_nb3;
    int n_q, n_kv, Hq, Hkv, G, B;
    int tok_per_tile, n_tiles_q, n_cta_q;
    int kv_bdiv;
    float qk_scale_log2;      // scale * log2(e)            (no softcap)
    float qk_scale, softcap;  // softcap path: softcap * tanh(raw * scale / softcap)
    float max_bias, m0, m1; int n_head_log2;
    int causal, window;
    int q_quant8;             // K was Q8_0: quantize Q rows like ggml's from_float
    int *err;
};

template <int D, int NQT> struct PrefillCfg {
    static constexpr int BM = 128, BN = 128;
    static constexpr int STAGES = D == 64 ? 3 : 2;
    static constexpr int SUB = D / 64;                         // 64-column swizzle sub-tiles
    static constexpr int TILE_BYTES = 128 * D * 2;             // one Q / K / V tile
    static constexpr int Q_OFF = 0;
    static constexpr int K_OFF = Q_OFF + NQT * TILE_BYTES;
    static constexpr int V_OFF = K_OFF + STAGES * TILE_BYTES;
    static constexpr int BAR_OFF = V_OFF + STAGES * TILE_BYTES;
    static constexpr int NBARS = 1 + 3 * STAGES + 2 * NQT + 1;
    static constexpr int SMEM = BAR_OFF + NBARS * 8 + 16 + 1024;   // +1024 alignment slack
    static constexpr int NTHREADS = 128 * NQT + 64;
    static constexpr int TMEM_USED = NQT * (128 + D);
    static constexpr int TMEM_COLS = TMEM_USED <= 256 ? 256 : 512;
    static constexpr int S_COL = 0;
    static constexpr int O_COL = NQT * 128;
};

// error codes written to PrefillArgs::err
enum { VTX_KERR_Q = 1, VTX_KERR_KV = 2, VTX_KERR_S = 3, VTX_KERR_P = 4, VTX_KERR_O = 5, VTX_KERR_EMPTY = 6 };

template <int D, int NQT, bool HAS_MASK>
__global__ void __launch_bounds__(PrefillCfg<D, NQT>::NTHREADS, 1)
fa_prefill_sm100_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                        const PrefillArgs a)
{
    using C = PrefillCfg<D, NQT>;
    extern __shared__ __align__(1024) char smem_raw[];
    char *smem = reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *q_full = bars;
    uint64_t *k_full = bars + 1;
    uint64_t *v_full = k_full + C::STAGES;
    uint64_t *kv_empty = v_full + C::STAGES;
    uint64_t *s_full = kv_empty + C::STAGES;
    uint64_t *p_full = s_full + NQT;
    uint64_t *o_full = p_full + NQT;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(o_full + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = blockIdx.y, b = blockIdx.z;
    const int qt0 = blockIdx.x * NQT;
    const int rows_per_tile = a.tok_per_tile * a.G;
    const int off = a.n_kv - a.n_q;

    // ---- key-tile range shared by all roles --------------------------------
    const int tok_first = qt0 * a.tok_per_tile;
    const int tok_last = min(a.n_q - 1, (min(qt0 + NQT, a.n_tiles_q)) * a.tok_per_tile - 1);
    int kv_lo = 0, kv_hi = a.n_kv - 1;
    if (a.causal) {
        kv_hi = min(kv_hi, tok_last + off);
        if (a.window > 0) kv_lo = max(0, tok_first + off - (a.window - 1));
    }
    const int j_begin = kv_lo / C::BN;
    const int j_end = kv_hi >= kv_lo ? kv_hi / C::BN + 1 : j_begin;
    const int n_iter = j_end - j_begin;

    if (tid == 0) {
        mbar_init(q_full, 128 * NQT);
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int t = 0; t < NQT; ++t) {
            mbar_init(&s_full[t], 1);
            mbar_init(&p_full[t], 128);
        }
        mbar_init(o_full, 1);
        fence_mbar_init();
    }
    if (warp == 4 * NQT + 1) {             // MMA warp owns the TMEM allocation
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    if (warp == 4 * NQT && lane == 0) {
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp < 4 * NQT) {
        // =================== softmax warpgroups ===============================
        const int t = warp >> 2;                   // Q tile within the CTA
        const int r = tid & 127;                   // row == TMEM lane
        const int qt = qt0 + t;
        const int tok = qt * a.tok_per_tile + r / a.G;
        const int head = g * a.G + r % a.G;
        const bool row_ok = qt < a.n_tiles_q && r < rows_per_tile && tok < a.n_q;
        int lo = 1, hi = 0;
        if (row_ok) {
            lo = 0;
            hi = a.n_kv - 1;
            if (a.causal) {
                hi = min(hi, tok + off);
                if (a.window > 0) lo = max(0, tok + off - (a.window - 1));
            }
        }
        // Q row -> f16 -> swizzled smem (K-major, 128B swizzle, 64-col sub-tiles)
        {
            char *qtile = smem + C::Q_OFF + t * C::TILE_BYTES;
            const char *src = a.q + (long long)tok * a.q_nb1 + (long long)head * a.q_nb2 + (long long)b * a.q_nb3;
            float qabs[D / 32];
#pragma unroll
            for (int i = 0; i < D / 32; ++i) qabs[i] = 0.0f;
            if (a.q_quant8 && row_ok) {
                for (int d = 0; d < D; ++d) {
                    const float x = a.q_f16 ? __half2float(reinterpret_cast<const __half *>(src)[d])
                                            : reinterpret_cast<const float *>(src)[d];
                    qabs[d >> 5] = fmaxf(qabs[d >> 5], fabsf(x));
                }
            }
#pragma unroll
            for (int c = 0; c < D / 8; ++c) {
                uint4 pk = make_uint4(0, 0, 0, 0);
                if (row_ok) {
                    float f[8];
                    if (a.q_f16) {
                        const uint4 raw = *reinterpret_cast<const uint4 *>(src + c * 16);
                        const __half2 *h = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
                        for (int i = 0; i < 4; ++i) { float2 x = __half22float2(h[i]); f[2 * i] = x.x; f[2 * i + 1] = x.y; }
                    } else {
                        const float4 x0 = *reinterpret_cast<const float4 *>(src + c * 32);
                        const float4 x1 = *reinterpret_cast<const float4 *>(src + c * 32 + 16);
                        f[0] = x0.x; f[1] = x0.y; f[2] = x0.z; f[3] = x0.w;
                        f[4] = x1.x; f[5] = x1.y; f[6] = x1.z; f[7] = x1.w;
                    }
                    if (a.q_quant8) {
                        // K is Q8_0 in the caller's tensor: ggml quantizes Q to Q8_0
                        // (per 32 values: d = amax/127, q = rne(x*127/amax)) before
                        // the dot; reproduce that and feed d*q (as half) to the MMA.
                        const int blk = c >> 2;
                        const float amax = qabs[blk];
                        const float dq = __half2float(__float2half_rn(amax / 127.0f));
                        const float id = amax != 0.0f ? 127.0f / amax : 0.0f;
#pragma unroll
                        for (int i = 0; i < 8; ++i) f[i] = dq * (float)__float2int_rn(f[i] * id);
                    }
                    pk.x = pack_half2(f[0], f[1]); pk.y = pack_half2(f[2], f[3]);
                    pk.z = pack_half2(f[4], f[5]); pk.w = pack_half2(f[6], f[7]);
                }
                const int sub = c >> 3, cc = c & 7;
                *reinterpret_cast<uint4 *>(qtile + sub * 16384 + r * 128 + ((cc ^ (r & 7)) << 4)) = pk;
            }
            fence_proxy_async_smem();
            mbar_arrive(q_full);
        }
        float slope = 1.0f;
        if (a.max_bias > 0.0f)
            slope = head < a.n_head_log2 ? powf(a.m0, (float)(head + 1))
                                         : powf(a.m1, (float)(2 * (head - a.n_head_log2) + 1));
        const char *mrow = nullptr;
        if (HAS_MASK && row_ok)
            mrow = a.mask + (long long)tok * a.m_nb1 + (long long)(head % a.m_ne2) * a.m_nb2 +
                   (long long)(b % a.m_ne3) * a.m_nb3;

        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t s_addr = tmem + lane_base + C::S_COL + t * 128;
        const uint32_t o_addr = tmem + lane_base + C::O_COL + t * D;
        float m_run = -INFINITY, l_run = 0.0f;

        for (int it = 0; it < n_iter && ok; ++it) {
            const int j = j_begin + it;
            ok = __all_sync(0xffffffffu, mbar_wait(&s_full[t], it & 1, a.err, VTX_KERR_S));
            if (!ok) break;
            tc_fence_after();
            float s[128];
            {
                uint32_t raw[128];
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    tmem_ld32(s_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&raw[c * 32]));
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 128; ++i) s[i] = __uint_as_float(raw[i]);
            }
            const int k0 = j * C::BN;
            const bool full = !HAS_MASK && k0 >= lo && k0 + C::BN - 1 <= hi;
            if (a.softcap != 0.0f) {
#pragma unroll
                for (int i = 0; i < 128; ++i) s[i] = a.softcap * tanhf(s[i] * a.qk_scale) * kLog2e;
            } else {
#pragma unroll
                for (int i = 0; i < 128; ++i) s[i] *= a.qk_scale_log2;
            }
            if (!full) {
#pragma unroll
                for (int i = 0; i < 128; ++i) {
                    const int key = k0 + i;
                    float x = s[i];
                    if (key < lo || key > hi) x = -INFINITY;
                    else if (HAS_MASK) {
                        const float mv = slope * __half2float(reinterpret_cast<const __half *>(mrow)[key]);
                        x = mv == -INFINITY ? -INFINITY : x + mv * kLog2e;
                    }
                    s[i] = x;
                }
            }
            float mx = s[0];
#pragma unroll
            for (int i = 1; i < 128; ++i) mx = fmaxf(mx, s[i]);
            bool rescale = false;
            float alpha = 1.0f;
            if (mx > m_run + 8.0f) {                 // lazy rescale: only on a 2^8 jump
                if (m_run != -INFINITY) {
                    alpha = ex2(m_run - mx);
                    rescale = it > 0;
                }
                m_run = mx;
                l_run *= alpha;
            }
            const float m_use = m_run == -INFINITY ? 0.0f : m_run;
            float sum = 0.0f;
#pragma unroll
            for (int i = 0; i < 128; ++i) {
                s[i] = ex2(s[i] - m_use);
                sum += s[i];
            }
            l_run += sum;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t pk[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) pk[i] = pack_half2(s[c * 64 + 2 * i], s[c * 64 + 2 * i + 1]);
                tmem_st32(s_addr + c * 32, pk);
            }
            // tcgen05.ld/st are warp-collective (.sync.aligned): the whole warp
            // rescales if any of its rows needs it (alpha == 1 for the others).
            if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
                for (int c = 0; c < D / 32; ++c) {
                    uint32_t o[32];
                    tmem_ld32(o_addr + c * 32, o);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_st32(o_addr + c * 32, o);
                }
            }
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(&p_full[t]);
        }
        // ---- epilogue: O / l -> dst ------------------------------------------
        if (ok && n_iter > 0) ok = __all_sync(0xffffffffu, mbar_wait(o_full, 0, a.err, VTX_KERR_O));
        if (ok) {
            tc_fence_after();
            float *out = reinterpret_cast<float *>(a.dst + (long long)tok * a.d_nb2 + (long long)head * a.d_nb1 +
                                                   (long long)b * a.d_nb3);
            const float inv = l_run == 0.0f ? 0.0f : 1.0f / l_run;
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
                uint32_t o[32];
                if (n_iter > 0) {
                    tmem_ld32(o_addr + c * 32, o);
                    tmem_ld_wait();
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = 0u;
                }
                if (row_ok) {
#pragma unroll
                    for (int i = 0; i < 32; i += 4) {
                        float4 v4 = make_float4(__uint_as_float(o[i]) * inv, __uint_as_float(o[i + 1]) * inv,
                                                __uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
                        *reinterpret_cast<float4 *>(out + c * 32 + i) = v4;
                    }
                }
            }
        }
    } else if (warp == 4 * NQT) {
        // =================== TMA producer =====================================
        if (lane == 0) {
            const int bkv = b / a.kv_bdiv;
            int issued = 0;
            for (int it = 0; it < n_iter; ++it) {
                const int st = it % C::STAGES;
                if (it >= C::STAGES &&
                    !mbar_wait(&kv_empty[st], ((it / C::STAGES) - 1) & 1, a.err, VTX_KERR_KV)) break;
                issued = it + 1;
                const int y = (j_begin + it) * C::BN;
                char *ks = smem + C::K_OFF + st * C::TILE_BYTES;
                char *vs = smem + C::V_OFF + st * C::TILE_BYTES;
                mbar_arrive_expect_tx(&k_full[st], C::TILE_BYTES);
#pragma unroll
                for (int sub = 0; sub < C::SUB; ++sub) tma_load_4d(ks + sub * 16384, &tmK, &k_full[st], sub * 64, y, g, bkv);
                mbar_arrive_expect_tx(&v_full[st], C::TILE_BYTES);
#pragma unroll
                for (int sub = 0; sub < C::SUB; ++sub) tma_load_4d(vs + sub * 16384, &tmV, &v_full[st], sub * 64, y, g, bkv);
            }
            // Drain: the last STAGES loads must have landed before this CTA's
            // shared memory can be released (already true unless a wait failed).
            for (int it = issued > C::STAGES ? issued - C::STAGES : 0; it < issued; ++it) {
                const int st = it % C::STAGES;
                mbar_wait(&k_full[st], (it / C::STAGES) & 1, a.err, VTX_KERR_KV);
                mbar_wait(&v_full[st], (it / C::STAGES) & 1, a.err, VTX_KERR_KV);
            }
        }
    } else {
        // =================== MMA issuer =======================================
        if (lane == 0 && n_iter > 0) {
            constexpr uint32_t IDESC_QK = idesc_f16_f32(128, 128, 0, 0);
            constexpr uint32_t IDESC_PV = idesc_f16_f32(128, D, 0, 1);
            const uint32_t sbase = smem_u32(smem);
            bool good = mbar_wait(q_full, 0, a.err, VTX_KERR_Q);
            tc_fence_after();
            for (int it = 0; it <= n_iter && good; ++it) {
                const int st = it % C::STAGES;
                const int pst = (it + C::STAGES - 1) % C::STAGES;
                if (it < n_iter) {
                    if (!mbar_wait(&k_full[st], (it / C::STAGES) & 1, a.err, VTX_KERR_KV)) { good = false; break; }
                }
                if (it > 0) {
                    if (!mbar_wait(&v_full[pst], ((it - 1) / C::STAGES) & 1, a.err, VTX_KERR_KV)) { good = false; break; }
                }
                tc_fence_after();
                for (int t = 0; t < NQT; ++t) {
                    const uint32_t s_tm = tmem + C::S_COL + t * 128;
                    if (it > 0) {
                        if (!mbar_wait(&p_full[t], (it - 1) & 1, a.err, VTX_KERR_P)) { good = false; break; }
                        tc_fence_after();
                        const uint32_t o_tm = tmem + C::O_COL + t * D;
                        const uint32_t vbase = sbase + C::V_OFF + pst * C::TILE_BYTES;
#pragma unroll
                        for (int kk = 0; kk < 8; ++kk) {
                            const uint64_t bdesc = smem_desc_sw128(vbase + kk * 2048, 16384, 1024);
                            mma_f16_ts(o_tm, s_tm + kk * 8, bdesc, IDESC_PV, (it > 1 || kk > 0) ? 1u : 0u);
                        }
                    }
                    if (it < n_iter) {
                        const uint32_t qbase = sbase + C::Q_OFF + t * C::TILE_BYTES;
                        const uint32_t kbase = sbase + C::K_OFF + st * C::TILE_BYTES;
#pragma unroll
                        for (int kk = 0; kk < D / 16; ++kk) {
                            const uint32_t koff = (kk >> 2) * 16384 + (kk & 3) * 32;
                            const uint64_t adesc = smem_desc_sw128(qbase + koff, 16, 1024);
                            const uint64_t bdesc = smem_desc_sw128(kbase + koff, 16, 1024);
                            mma_f16_ss(s_tm, adesc, bdesc, IDESC_QK, kk > 0 ? 1u : 0u);
                        }
                        mma_commit(&s_full[t]);
                    }
                }
                if (!good) break;
                if (it > 0) mma_commit(&kv_empty[pst]);
            }
            mma_commit(o_full);
            // every MMA of this CTA must be retired before TMEM is released
            mbar_wait(o_full, 0, a.err, VTX_KERR_O);
        }
    }

    // ---- teardown -------------------------------------------------------------
    tc_fence_before();
    __syncthreads();
    if (warp == 4 * NQT + 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

}  // namespace vtx
