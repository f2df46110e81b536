// sm_100a device code of the int8 engine.
//
//   conv_tc_kernel   implicit-GEMM conv: TMA (4-D tiled, element strides for
//                    stride-2, out-of-bounds zero fill = padding code 0) ->
//                    tcgen05.mma kind::i8 (int32 accumulators in TMEM) ->
//                    fused exact epilogue (dequant, bias, act, residual add,
//                    requant to int8 codes for every consumer scale).
//   stem_im2col      fp32 NCHW network input -> exact int8 codes in im2col rows
//                    (K = kh*kw*cin padded to 32), so the stem runs as a 1x1
//                    GEMM through conv_tc_kernel.
//   dw_conv_kernel   depthwise kxk conv over int8 NHWC codes (memory bound).
//   maxpool_kernel   3x3/s2/p1 maxpool of the fp32 stem output + requant.
//   head_kernel      global average pool + FC.
//
// Numeric contract (bit-exact with the reference integer oracle,
// 09-ptq-toolkit/ptq_toolkit/ref_int8.py:89-91,218-250):
//   codes = clip(round_half_away(double(x) / s), -128, 127), s a double;
//   y = fadd(fmul(float(acc), factor[c]), bias[c])  (two roundings, no FMA);
//   factor[c] = float(float(s_in) * w_scale[c]) is precomputed on the host.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ptq8 {

// Sticky device error word: a bounded wait that ran out records where.
__device__ int g_ptq8_error;

enum : int {
    ERR_NONE = 0,
    ERR_WAIT_EMPTY = 1,
    ERR_WAIT_FULL = 2,
    ERR_WAIT_ACC = 3,
    ERR_DRAIN = 4,
};

// About 2 s at the B200 boost clock; no wait in these kernels is expected to
// take more than microseconds.
constexpr long long kWaitLimitCycles = 4000000000LL;

// ------------------------------------------------------------------ PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    if (mbar_try(bar, parity)) return true;
    const long long t0 = clock64();
    while (true) {
        if (mbar_try(bar, parity)) return true;
        if (clock64() - t0 > kWaitLimitCycles) return false;
    }
}

__device__ __forceinline__ void tma_prefetch(const CUtensorMap* m) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* m, uint32_t bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* m, uint32_t bar, int c0, int c1,
                                            int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, signed int8 -> int32.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on an mbarrier once every previously issued tcgen05.mma of this thread completes.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32"
        " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
        " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
          "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
          "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
          "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand tile whose rows are
// `cb` bytes long and stored with the matching TMA swizzle (cb = 32/64/128):
// 8-row core groups `8*cb` bytes apart (SBO), LBO unused for swizzled K-major.
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, int cb) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>(1) << 16;
    d |= static_cast<uint64_t>((8u * cb) >> 4) << 32;
    d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
    const uint64_t layout = cb == 128 ? 2u : (cb == 64 ? 4u : 6u);
    d |= layout << 61;
    return d;
}

// Instruction descriptor: kind::i8, D = s32, A = B = s8, both K-major, M = 128.
__host__ __device__ constexpr uint32_t make_idesc_i8(int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(128 >> 4) << 24);
}

// ------------------------------------------------------------------ exact quantize

// Exact int8 code of x for scale s (s64) with inv = float(1/s):
// clip(round_half_away(double(x)/s), -128, 127).  The float estimate t = x*inv
// is within 2e-5 of x/s for |x/s| <= 129; whenever t is more than 1e-4 away
// from a half-integer its nearest integer is the reference's code, otherwise
// the reference's double-precision formula is evaluated.
__device__ __forceinline__ int quant_code(float x, float inv, double s) {
    const float t = __fmul_rn(x, inv);
    const float r = rintf(t);
    if (fabsf(__fsub_rn(t, r)) < 0.4999f) {
        return static_cast<int>(fminf(fmaxf(r, -128.0f), 127.0f));
    }
    const double v = static_cast<double>(x) / s;
    double q = v >= 0.0 ? floor(v + 0.5) : ceil(v - 0.5);
    q = fmin(fmax(q, -128.0), 127.0);
    return static_cast<int>(q);
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
    return (static_cast<uint32_t>(a) & 0xFFu) | ((static_cast<uint32_t>(b) & 0xFFu) << 8) |
           ((static_cast<uint32_t>(c) & 0xFFu) << 16) | ((static_cast<uint32_t>(d) & 0xFFu) << 24);
}

__device__ __forceinline__ float apply_act(float y, int act) {
    if (act == 1) return fmaxf(y, 0.0f);
    if (act == 2) return fminf(fmaxf(y, 0.0f), 6.0f);
    return y;
}

// ------------------------------------------------------------------ epilogue outputs

struct EpiParams {
    const float* factor;    // [cout] float(float(s_in) * w_scale[c])
    const float* bias;      // [cout]
    const float* residual;  // fp32 NHWC [P][cout] or null
    float* out_f32;         // fp32 NHWC [P][cout] or null
    int8_t* out_q0;         // int8 NHWC codes [P][ldq0] or null
    int8_t* out_q1;
    int ldq0, ldq1;
    float inv0, inv1;
    double s0, s1;
    int cout;
    int act;   // activation of the conv itself: 0 none / 1 relu / 2 relu6
    int post;  // residual: 0 none, 1 add then relu, 2 add only
};

// Finish 32 consecutive channels [c0, c0+32) of output position p (nv of them valid).
__device__ __forceinline__ void epilogue_store32(const EpiParams& e, size_t p, int c0, int nv, float (&y)[32]) {
    if (e.post != 0) {
        const float* rp = e.residual + p * e.cout + c0;
        if (nv == 32) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
                float4 r = __ldg(reinterpret_cast<const float4*>(rp + j));
                y[j] = __fadd_rn(y[j], r.x);
                y[j + 1] = __fadd_rn(y[j + 1], r.y);
                y[j + 2] = __fadd_rn(y[j + 2], r.z);
                y[j + 3] = __fadd_rn(y[j + 3], r.w);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < nv) y[j] = __fadd_rn(y[j], rp[j]);
        }
        if (e.post == 1) {
#pragma unroll
            for (int j = 0; j < 32; ++j) y[j] = fmaxf(y[j], 0.0f);
        }
    }
    if (e.out_f32) {
        float* op = e.out_f32 + p * e.cout + c0;
        if (nv == 32) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
                *reinterpret_cast<float4*>(op + j) = make_float4(y[j], y[j + 1], y[j + 2], y[j + 3]);
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < nv) op[j] = y[j];
        }
    }
#pragma unroll
    for (int o = 0; o < 2; ++o) {
        int8_t* qbase = o == 0 ? e.out_q0 : e.out_q1;
        if (!qbase) continue;
        const float inv = o == 0 ? e.inv0 : e.inv1;
        const double s = o == 0 ? e.s0 : e.s1;
        int8_t* qp = qbase + p * static_cast<size_t>(o == 0 ? e.ldq0 : e.ldq1) + c0;
        if (nv == 32) {
            uint32_t w[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                w[j] = pack4(quant_code(y[4 * j], inv, s), quant_code(y[4 * j + 1], inv, s),
                             quant_code(y[4 * j + 2], inv, s), quant_code(y[4 * j + 3], inv, s));
            reinterpret_cast<uint4*>(qp)[0] = make_uint4(w[0], w[1], w[2], w[3]);
            reinterpret_cast<uint4*>(qp)[1] = make_uint4(w[4], w[5], w[6], w[7]);
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < nv) qp[j] = static_cast<int8_t>(quant_code(y[j], inv, s));
        }
    }
}

// ------------------------------------------------------------------ tensor-core conv

struct ConvGeom {
    int N, OH, OW;              // output map (per image)
    int TW, TH, TN;             // one M tile = TN images x TH rows x TW cols (<= 128 positions)
    int tiles_w, tiles_h;       // M tiles along W and H
    int KW, SH, SW, PH, PW;     // kernel width, strides, paddings
    int n_cchunks, n_kchunks;   // channel chunks per tap, total K chunks
    int BN;                     // N tile (multiple of 16, <= 256)
    int tmem_cols;              // power of two >= max(32, BN)
    uint32_t a_bytes, b_bytes;  // TMA bytes per stage
};

constexpr int kConvThreads = 192;   // warp 0 TMA, warp 1 MMA, warps 2..5 epilogue

template <int CB, int STAGES>
__global__ void __launch_bounds__(kConvThreads, 1)
conv_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
               const ConvGeom g, const EpiParams e) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ int s_abort;
    // A wait of an earlier CTA already ran out: skip the work (block-uniform decision).
    if (threadIdx.x == 0) s_abort = *reinterpret_cast<volatile int*>(&g_ptq8_error);
    __syncthreads();
    if (s_abort) return;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int BN = g.BN;
    const int bn32 = (BN + 31) & ~31;
    const int sb_stride = (BN * CB + 1023) & ~1023;   // every stage 1024-byte aligned (swizzle atoms)
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * 128 * CB;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sB + STAGES * sb_stride);  // full[S], empty[S], acc
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 1);
    float* s_factor = reinterpret_cast<float*>(tslot + 4);
    float* s_bias = s_factor + bn32;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int mt = blockIdx.x;
    const int nt = blockIdx.y;
    const int tw_i = mt % g.tiles_w;
    const int rest = mt / g.tiles_w;
    const int th_i = rest % g.tiles_h;
    const int tn_i = rest / g.tiles_h;
    const int w0 = tw_i * g.TW, h0 = th_i * g.TH, n0 = tn_i * g.TN;

    const uint32_t full0 = smem_u32(bars);
    const uint32_t empty0 = smem_u32(bars + STAGES);
    const uint32_t accbar = smem_u32(bars + 2 * STAGES);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        mbar_init(accbar, 1);
        fence_mbar_init();
        tma_prefetch(&map_a);
        tma_prefetch(&map_b);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tslot), g.tmem_cols);
        tmem_relinquish();
    }
    if (warp >= 2) {
        for (int c = threadIdx.x - 64; c < bn32; c += 128) {
            const int gc = nt * BN + c;
            const bool ok = c < BN && gc < e.cout;
            s_factor[c] = ok ? e.factor[gc] : 0.0f;
            s_bias[c] = ok ? e.bias[gc] : 0.0f;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer
            int issued = 0;
            for (int kc = 0; kc < g.n_kchunks; ++kc) {
                const int s = kc % STAGES;
                const uint32_t ph = (kc / STAGES) & 1;
                if (!mbar_wait(empty0 + 8 * s, ph ^ 1)) {
                    atomicExch(&g_ptq8_error, ERR_WAIT_EMPTY);
                    break;
                }
                const int tap = kc / g.n_cchunks;
                const int cc = kc - tap * g.n_cchunks;
                const int ki = tap / g.KW;
                const int kj = tap - ki * g.KW;
                mbar_expect_tx(full0 + 8 * s, g.a_bytes + g.b_bytes);
                tma_load_4d(smem_u32(sA + s * 128 * CB), &map_a, full0 + 8 * s, cc * CB, w0 * g.SW + kj - g.PW,
                            h0 * g.SH + ki - g.PH, n0);
                tma_load_2d(smem_u32(sB + s * sb_stride), &map_b, full0 + 8 * s, kc * CB, nt * BN);
                issued = kc + 1;
            }
            // Drain: every issued copy must have landed before the CTA can exit.
            for (int kc = issued > STAGES ? issued - STAGES : 0; kc < issued; ++kc) {
                if (!mbar_wait(full0 + 8 * (kc % STAGES), (kc / STAGES) & 1)) {
                    atomicExch(&g_ptq8_error, ERR_DRAIN);
                    break;
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer
            const uint32_t idesc = make_idesc_i8(BN);
            for (int kc = 0; kc < g.n_kchunks; ++kc) {
                const int s = kc % STAGES;
                if (!mbar_wait(full0 + 8 * s, (kc / STAGES) & 1)) {
                    atomicExch(&g_ptq8_error, ERR_WAIT_FULL);
                    break;
                }
                tc_fence_after();
                const uint64_t da = make_sdesc(smem_u32(sA + s * 128 * CB), CB);
                const uint64_t db = make_sdesc(smem_u32(sB + s * sb_stride), CB);
#pragma unroll
                for (int k = 0; k < CB / 32; ++k)
                    mma_i8(tmem, da + 2 * k, db + 2 * k, idesc, (kc | k) != 0 ? 1u : 0u);
                mma_commit(empty0 + 8 * s);
            }
            mma_commit(accbar);
        }
    } else {
        // ---------------- epilogue: TMEM lanes 32*(warp%4) .. +31 = tile rows
        const int quad = warp & 3;
        const int r = quad * 32 + lane;
        const int tw = g.TW, th = g.TH;
        const int n = n0 + r / (tw * th);
        const int h = h0 + (r / tw) % th;
        const int w = w0 + r % tw;
        const bool valid = r < tw * th * g.TN && n < g.N && h < g.OH && w < g.OW;
        const size_t p = (static_cast<size_t>(n) * g.OH + h) * g.OW + w;
        const bool ok = mbar_wait(accbar, 0);
        if (!ok) atomicExch(&g_ptq8_error, ERR_WAIT_ACC);
        tc_fence_after();
        const int tile_end = min(e.cout, (nt + 1) * BN);
        for (int cg = 0; cg < bn32 / 32; ++cg) {
            uint32_t v[32];
            tmem_ld32(tmem + (static_cast<uint32_t>(quad * 32) << 16) + cg * 32, v);
            tmem_wait_ld();
            const int c0 = nt * BN + cg * 32;
            if (!ok || !valid || c0 >= tile_end) continue;
            const int nv = min(32, tile_end - c0);
            float y[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const float a = static_cast<float>(static_cast<int>(v[j]));
                y[j] = apply_act(__fadd_rn(__fmul_rn(a, s_factor[cg * 32 + j]), s_bias[cg * 32 + j]), e.act);
            }
            epilogue_store32(e, p, c0, nv, y);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, g.tmem_cols);
}

// ------------------------------------------------------------------ stem im2col

// x: fp32 NCHW [N][C][H][W]; out: int8 [N*OH*OW][kpad] with k = (i*KW + j)*C + c,
// codes of the stem's scale, zero for out-of-image taps and k >= KH*KW*C.
__global__ void stem_im2col_kernel(const float* __restrict__ x, int8_t* __restrict__ out, int N, int C, int H,
                                   int W, int OH, int OW, int KH, int KW, int SH, int SW, int PH, int PW,
                                   int kpad, float inv, double s) {
    const size_t rows = static_cast<size_t>(N) * OH * OW;
    const int words = kpad / 4;
    for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < rows * words;
         idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t row = idx / words;
        const int wd = static_cast<int>(idx - row * words);
        const int ow = static_cast<int>(row % OW);
        const int oh = static_cast<int>((row / OW) % OH);
        const int n = static_cast<int>(row / (static_cast<size_t>(OW) * OH));
        int q[4];
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int k = wd * 4 + b;
            q[b] = 0;
            if (k < KH * KW * C) {
                const int c = k % C;
                const int tap = k / C;
                const int i = tap / KW, j = tap % KW;
                const int ih = oh * SH + i - PH, iw = ow * SW + j - PW;
                if (ih >= 0 && ih < H && iw >= 0 && iw < W)
                    q[b] = quant_code(__ldg(x + ((static_cast<size_t>(n) * C + c) * H + ih) * W + iw), inv, s);
            }
        }
        reinterpret_cast<uint32_t*>(out)[idx] = pack4(q[0], q[1], q[2], q[3]);
    }
}

// ------------------------------------------------------------------ depthwise conv

// Depthwise kxk conv over int8 NHWC codes [N][H][W][ldi] (C channels), int32
// accumulation, then the shared exact epilogue.  One thread per (position,
// 4 channels); weights w[tap][C] int8.
__global__ void dw_conv_kernel(const int8_t* __restrict__ in, int ldi, const int8_t* __restrict__ w, int N, int H,
                               int W, int C, int OH, int OW, int KH, int KW, int SH, int SW, int PH, int PW,
                               const EpiParams e) {
    const int cq = (C + 3) / 4;
    const size_t total = static_cast<size_t>(N) * OH * OW * cq;
    for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int c4 = static_cast<int>(idx % cq);
        const size_t p = idx / cq;
        const int ow = static_cast<int>(p % OW);
        const int oh = static_cast<int>((p / OW) % OH);
        const int n = static_cast<int>(p / (static_cast<size_t>(OW) * OH));
        const int c0 = c4 * 4;
        int acc[4] = {0, 0, 0, 0};
        for (int i = 0; i < KH; ++i) {
            const int ih = oh * SH + i - PH;
            if (ih < 0 || ih >= H) continue;
            for (int j = 0; j < KW; ++j) {
                const int iw = ow * SW + j - PW;
                if (iw < 0 || iw >= W) continue;
                const char4 xv = *reinterpret_cast<const char4*>(in + ((static_cast<size_t>(n) * H + ih) * W + iw) * ldi + c0);
                const int8_t* wr = w + static_cast<size_t>(i * KW + j) * C + c0;
                acc[0] += static_cast<int>(xv.x) * wr[0];
                if (c0 + 1 < C) acc[1] += static_cast<int>(xv.y) * wr[1];
                if (c0 + 2 < C) acc[2] += static_cast<int>(xv.z) * wr[2];
                if (c0 + 3 < C) acc[3] += static_cast<int>(xv.w) * wr[3];
            }
        }
        const int nv = min(4, C - c0);
        float y[4];
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int c = min(c0 + b, C - 1);
            y[b] = apply_act(__fadd_rn(__fmul_rn(static_cast<float>(acc[b]), e.factor[c]), e.bias[c]), e.act);
        }
        if (e.post != 0) {
            for (int b = 0; b < nv; ++b) {
                y[b] = __fadd_rn(y[b], e.residual[p * C + c0 + b]);
                if (e.post == 1) y[b] = fmaxf(y[b], 0.0f);
            }
        }
        if (e.out_f32)
            for (int b = 0; b < nv; ++b) e.out_f32[p * C + c0 + b] = y[b];
        if (e.out_q0)
            for (int b = 0; b < nv; ++b) e.out_q0[p * e.ldq0 + c0 + b] = static_cast<int8_t>(quant_code(y[b], e.inv0, e.s0));
        if (e.out_q1)
            for (int b = 0; b < nv; ++b) e.out_q1[p * e.ldq1 + c0 + b] = static_cast<int8_t>(quant_code(y[b], e.inv1, e.s1));
    }
}

// ------------------------------------------------------------------ stem maxpool

// 3x3/s2/p1 maxpool (padding never wins) of fp32 NHWC [N][H][W][C]; writes the
// pooled fp32 map and its codes.  Quantization is monotone, so pooling the fp32
// values and then quantizing equals the reference's order (ref_e2e.py:192-203).
__global__ void maxpool_kernel(const float* __restrict__ in, int N, int H, int W, int C, int OH, int OW,
                               const EpiParams e) {
    const size_t total = static_cast<size_t>(N) * OH * OW * C;
    for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(idx % C);
        const size_t p = idx / C;
        const int ow = static_cast<int>(p % OW);
        const int oh = static_cast<int>((p / OW) % OH);
        const int n = static_cast<int>(p / (static_cast<size_t>(OW) * OH));
        float m = -INFINITY;
        for (int i = 0; i < 3; ++i) {
            const int ih = oh * 2 + i - 1;
            if (ih < 0 || ih >= H) continue;
            for (int j = 0; j < 3; ++j) {
                const int iw = ow * 2 + j - 1;
                if (iw < 0 || iw >= W) continue;
                m = fmaxf(m, in[((static_cast<size_t>(n) * H + ih) * W + iw) * C + c]);
            }
        }
        if (e.out_f32) e.out_f32[p * C + c] = m;
        if (e.out_q0) e.out_q0[p * e.ldq0 + c] = static_cast<int8_t>(quant_code(m, e.inv0, e.s0));
        if (e.out_q1) e.out_q1[p * e.ldq1 + c] = static_cast<int8_t>(quant_code(m, e.inv1, e.s1));
    }
}

// ------------------------------------------------------------------ head

// logits[n][o] = fc_b[o] + sum_c fc_w[o][c] * mean_p x[n][p][c]
// One CTA per image: fixed-order fp32 position sums, float64 FC accumulation.
__global__ void head_kernel(const float* __restrict__ x, int HW, int C, const float* __restrict__ fc_w,
                            const float* __restrict__ fc_b, int n_out, float* __restrict__ logits) {
    extern __shared__ float pooled[];
    const int n = blockIdx.x;
    const float* xn = x + static_cast<size_t>(n) * HW * C;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        float s = 0.0f;
        for (int p = 0; p < HW; ++p) s = __fadd_rn(s, xn[static_cast<size_t>(p) * C + c]);
        pooled[c] = __fdiv_rn(s, static_cast<float>(HW));
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int o = warp; o < n_out; o += nw) {
        double acc = 0.0;
        for (int c = lane; c < C; c += 32) acc += static_cast<double>(fc_w[static_cast<size_t>(o) * C + c]) * pooled[c];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        if (lane == 0) logits[static_cast<size_t>(n) * n_out + o] = static_cast<float>(acc + static_cast<double>(fc_b[o]));
    }
}

}  // namespace ptq8
