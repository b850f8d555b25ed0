// out_proj.cuh — the attention output projection on tcgen05 (sm_100a).
//
// voxtral.cpp follows each attention node with
//     attn_out  = ggml_cont(attn_out)                      // [Dv*Hq, n]
//     attn_proj = ggml_mul_mat(attn_o_weight, attn_out)    // [dim, n]
//     (+ attn_o_bias, encoder only)  then  x = residual + attn_proj
// (src/voxtral.cpp:1612-1617 encoder, :1804-1809 decoder).  Here that is one
// kernel: Y[t][n] = residual[t][n] + bias[n] + sum_k A[t][k] W[n][k], with A
// the attention's F32 output read in place (no contiguous copy) and W the
// F16 weight as ggml stores it ([K] rows, one per output feature).
//
// One CTA per 128 x 128 output tile, K in steps of 64:
//   warp 0       TMA producer: per K step one box of A (64 F32 columns x 128
//                tokens, unswizzled) and one of W (64 f16 x 128 rows, 128-byte
//                swizzle) into a STAGES-deep ring;
//   warps 2-5    convert each A box to f16 (round to nearest even, as ggml
//                rounds activations for an F16 weight) in the 128-byte
//                swizzled K-major layout the MMA reads; after the last K
//                step they run the epilogue;
//   warp 1       MMA issuer: D[128 x 128] (TMEM, f32) += A16 * W^T, four
//                tcgen05.mma (K = 16) per step, stage released by commit.
// Epilogue: the four warps read their 32 TMEM lanes (tokens) 32 columns at a
// time, add bias and residual, stage the box in the output map's 128-byte
// swizzle and write it with a TMA store (two staging buffers in turn).
//
// With an F16 A (the attention written with an F16 result, the same rounding
// done once upstream) the A boxes land by TMA in the MMA's swizzled layout:
// no conversion warps, half the A bytes, four stages instead of three and the
// residual tile fetched into its own buffer while the K loop runs.
//
// A is addressed as [Dv, H_in, n, H_out] so a head-split result gathered by
// rank (head h = r * H_in + j, each rank's block at its own stride) is read
// as is.  K = Hq * Dv must be a multiple of 64, Dv a multiple of 64.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "vtx_ptx.cuh"

namespace vtx {

struct OutProjArgs {
    int M, N, K;            // tokens, output features, Hq * Dv
    int Dv, h_in;           // head size; heads per block of A (head h = h / h_in block, h % h_in inside)
    const float *bias;      // [N] or null
    const char *res;        // residual rows (F32, stride res_nb1 bytes) or null
    long long res_nb1;
    int *err;
};

// AF16: the attention output is already F16 (the rounding ggml applies to the
// activations of an F16-weight mat-mul, done in the attention epilogue): A
// boxes land by TMA in the MMA's 128-byte swizzled layout, no conversion, half
// the bytes per stage.
template <bool AF16 = false> struct OutProjCfgT {
    static constexpr int BM = 128, BN = 128, BK = 64, STAGES = AF16 ? 4 : 3;
    static constexpr int A32_BYTES = AF16 ? 0 : BM * BK * 4;    // 32 KB F32 box
    static constexpr int A16_BYTES = BM * BK * 2;               // 16 KB f16, swizzled
    static constexpr int W_BYTES = BN * BK * 2;                 // 16 KB f16, swizzled
    static constexpr int STAGE = A32_BYTES + A16_BYTES + W_BYTES;
    static constexpr int OUT_BOX = BM * 32 * 4;                 // [128 tokens][32 floats]
    static constexpr int OUT_OFF = STAGES * STAGE;
    // AF16: the residual tile has its own buffer and is fetched while the K
    // loop runs (the conversion warps are idle); F32 A: it is fetched into the
    // freed stages once every MMA has retired.  The tile's bias columns are
    // staged in shared memory before the epilogue in both cases.
    static constexpr int RES_OFF = OUT_OFF + 2 * OUT_BOX;
    static constexpr int BIAS_OFF = RES_OFF + (AF16 ? BN / 32 * OUT_BOX : 0);
    static constexpr int BAR_OFF = BIAS_OFF + BN * 4;
    // full[S], conv[S], empty[S], acc, res_full
    static constexpr int NBARS = 3 * STAGES + 2;
    static_assert(BN / 32 * OUT_BOX <= STAGES * STAGE, "the residual tile fits in the freed stages");
    static constexpr int SMEM = BAR_OFF + NBARS * 8 + 16 + 1024;
    static constexpr int NTHREADS = 192;
    static constexpr int TMEM_COLS = 128;
};
using OutProjCfg = OutProjCfgT<false>;

template <bool AF16>
__global__ void __launch_bounds__(OutProjCfgT<AF16>::NTHREADS, 1)
out_proj_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                const __grid_constant__ CUtensorMap tmY, const __grid_constant__ CUtensorMap tmR,
                const OutProjArgs a)
{
    using C = OutProjCfgT<AF16>;
    constexpr int ST = C::STAGES;
    extern __shared__ __align__(1024) char smem_raw[];
    char *smem = reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *full = bars;                  // [ST] A32 and W of a stage landed
    uint64_t *conv = full + ST;             // [ST] A16 of a stage written (4 warp arrivals)
    uint64_t *empty = conv + ST;            // [ST] the stage's MMAs retired
    uint64_t *acc = empty + ST;             // every MMA retired
    uint64_t *res_full = acc + 1;           // the residual tile landed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(res_full + 1);
    auto a32 = [&](int s) { return smem + s * C::STAGE; };
    auto a16 = [&](int s) { return smem + s * C::STAGE + C::A32_BYTES; };
    auto wt = [&](int s) { return smem + s * C::STAGE + C::A32_BYTES + C::A16_BYTES; };

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.x * C::BM, n0 = blockIdx.y * C::BN;
    const int nk = a.K / C::BK;

    if (tid == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&conv[s], 4);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc, 1);
        mbar_init(res_full, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmW);
        tma_prefetch_desc(&tmY);
        if (a.res) tma_prefetch_desc(&tmR);
    }
    grid_dep_wait();
    grid_dep_launch();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // =================== TMA producer =====================================
        if (lane == 0) {
            int issued = 0;
            for (int i = 0; i < nk; ++i) {
                const int s = i % ST;
                if (i >= ST && !mbar_wait(&empty[s], (uint32_t)(((i / ST) - 1) & 1), a.err, VTX_KERR_KV)) break;
                const int k0 = i * C::BK;
                const int h = k0 / a.Dv, d0 = k0 % a.Dv;
                mbar_arrive_expect_tx(&full[s], (AF16 ? C::A16_BYTES : C::A32_BYTES) + C::W_BYTES);
                tma_load_4d(AF16 ? a16(s) : a32(s), &tmA, &full[s], d0, h % a.h_in, m0, h / a.h_in);
                tma_load_2d(wt(s), &tmW, &full[s], k0, n0);
                issued = i + 1;
            }
            for (int i = issued > ST ? issued - ST : 0; i < issued; ++i)
                mbar_wait(&full[i % ST], (uint32_t)((i / ST) & 1), a.err, VTX_KERR_KV);
        }
    } else if (warp == 1) {
        // =================== MMA issuer =======================================
        const uint32_t lead = elect_one();
        constexpr uint32_t IDESC = idesc_f16_f32(128, C::BN, 0, 0);
        constexpr uint32_t HI = (1024u >> 4) | (1u << 14) | (2u << 29);   // SBO 1024, v1, SW128
        bool good = true;
        for (int i = 0; i < nk && good; ++i) {
            const int s = i % ST;
            // F32 A: wait for the conversion; F16 A: for the TMA loads themselves
            good = __all_sync(0xffffffffu, mbar_wait(AF16 ? &full[s] : &conv[s], (uint32_t)((i / ST) & 1), a.err,
                                                     VTX_KERR_Q));
            if (!good) break;
            tc_fence_after();
            const uint32_t alo = (smem_u32(a16(s)) >> 4) | (1u << 16);
            const uint32_t blo = (smem_u32(wt(s)) >> 4) | (1u << 16);
#pragma unroll
            for (int kk = 0; kk < C::BK / 16; ++kk)
                mma_f16_ss_w(lead, tmem, desc64(alo + kk * 2, HI), desc64(blo + kk * 2, HI), IDESC,
                             (i > 0 || kk > 0) ? 1u : 0u);
            mma_commit_w(lead, &empty[s]);
        }
        mma_commit_w(lead, acc);
        mbar_wait(acc, 0, a.err, VTX_KERR_O);
    } else {
        // =================== convert A, then the epilogue ====================
        const int t = tid - 64;                        // 0..127
        bool ok = true;
        for (int i = 0; i < (AF16 ? 0 : nk) && ok; ++i) {
            const int s = i % ST;
            ok = __all_sync(0xffffffffu, mbar_wait(&full[s], (uint32_t)((i / ST) & 1), a.err, VTX_KERR_KV));
            if (!ok) break;
            const char *src = a32(s);
            char *dst = a16(s);
            // warp q converts rows 32q .. 32q + 31, two rows (512 contiguous
            // bytes, conflict-free) per instruction: lane l takes floats
            // 4 (l % 16) .. + 3 of row 2 it + l / 16 and writes their halves
            // as one 8-byte half of a swizzled 16-byte chunk (a half-warp
            // writes one whole 128-byte row: conflict-free as well)
            const int q = t >> 5, f4 = lane & 15;
#pragma unroll 4
            for (int it = 0; it < 16; ++it) {
                const int row = 32 * q + 2 * it + (lane >> 4);
                const float4 x = *reinterpret_cast<const float4 *>(src + row * 256 + f4 * 16);
                *reinterpret_cast<uint2 *>(dst + row * 128 + (((f4 >> 1) ^ (row & 7)) << 4) + (f4 & 1) * 8) =
                    make_uint2(pack_half2(x.x, x.y), pack_half2(x.z, x.w));
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&conv[s]);
        }
        const bool leader = warp == 2 && lane == 0;
        char *res_tile = AF16 ? smem + C::RES_OFF : smem;
        if (AF16 && a.res && leader) {                 // the residual tile, while the K loop runs
            mbar_arrive_expect_tx(res_full, C::BN / 32 * C::OUT_BOX);
#pragma unroll
            for (int c = 0; c < C::BN / 32; ++c) tma_load_2d(res_tile + c * C::OUT_BOX, &tmR, res_full, n0 + c * 32, m0);
        }
        float *bias_s = reinterpret_cast<float *>(smem + C::BIAS_OFF);
        if (a.bias) bias_s[t] = n0 + t < a.N ? __ldg(a.bias + n0 + t) : 0.0f;
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(acc, 0, a.err, VTX_KERR_O));
        tc_fence_after();
        // this warp's TMEM lanes: tokens 32q .. 32q + 31 of the tile
        const int q = warp & 3, r = 32 * q + lane;
        const uint32_t t_row = tmem + ((uint32_t)(32 * q) << 16);
        // F32 A: every MMA has retired and every load has landed (the MMA
        // consumed them), so the stage buffers are free: the whole residual
        // tile is fetched into them at once, in the output boxes' swizzled layout.
        if (!AF16 && a.res && leader && ok) {
            mbar_arrive_expect_tx(res_full, C::BN / 32 * C::OUT_BOX);
#pragma unroll
            for (int c = 0; c < C::BN / 32; ++c) tma_load_2d(res_tile + c * C::OUT_BOX, &tmR, res_full, n0 + c * 32, m0);
        }
        // (AF16: waited even after a failed wait above: the load was issued and
        // must land before the CTA's shared memory is released)
        if (a.res && (ok || AF16)) ok = __all_sync(0xffffffffu, mbar_wait(res_full, 0, a.err, VTX_KERR_O)) && ok;
        for (int c = 0; c < C::BN / 32; ++c) {
            char *stg = smem + C::OUT_OFF + (c & 1) * C::OUT_BOX;
            if (c >= 2 && leader) bulk_wait_read<1>();   // the store that used this buffer has read it
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (ok) {
                uint32_t v[32];
                tmem_ld32(t_row + c * 32, v);
                tmem_ld_wait();
                float f[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(v[i]);
                if (a.bias) {                   // staged above; 0 past the tensor
#pragma unroll
                    for (int i = 0; i < 32; ++i) f[i] += bias_s[c * 32 + i];
                }
                if (a.res) {                    // rows / columns past the tensor read as zeros
                    const char *rb = res_tile + c * C::OUT_BOX + r * 128;
#pragma unroll
                    for (int q4 = 0; q4 < 8; ++q4) {
                        const float4 x = *reinterpret_cast<const float4 *>(rb + ((q4 ^ (r & 7)) << 4));
                        f[4 * q4] += x.x; f[4 * q4 + 1] += x.y; f[4 * q4 + 2] += x.z; f[4 * q4 + 3] += x.w;
                    }
                }
#pragma unroll
                for (int q4 = 0; q4 < 8; ++q4)
                    *reinterpret_cast<float4 *>(stg + r * 128 + ((q4 ^ (r & 7)) << 4)) =
                        make_float4(f[4 * q4], f[4 * q4 + 1], f[4 * q4 + 2], f[4 * q4 + 3]);
            }
            fence_proxy_async_smem();
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (leader && ok) {
                tma_store_2d_f32(&tmY, stg, n0 + c * 32, m0);
                bulk_commit();
            }
        }
        if (leader) bulk_wait_all_done();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

}  // namespace vtx
