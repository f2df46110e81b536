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

#include <cmath>

namespace ptq8 {

// Codes a bounded wait that ran out records in its engine's device error word
// (an int in engine-owned device memory, passed to every kernel that waits, so
// one engine's timeout never aborts another engine's kernels).
enum : int {
    ERR_NONE = 0,
    ERR_WAIT_EMPTY = 1,
    ERR_WAIT_FULL = 2,
    ERR_WAIT_ACC = 3,
    ERR_DRAIN = 4,
};

// Default wait limit: about 2 s at the B200 boost clock; no wait in these
// kernels is expected to take more than microseconds.
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

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Arrive without release semantics.  The epilogue frees a TMEM accumulator
// this way: the only accesses to order are its tcgen05.ld reads (completed by
// tcgen05.wait::ld and ordered by tcgen05.fence::before_thread_sync); a release
// arrive would also wait for the warp's outstanding global stores to reach the
// point of coherence and put that latency on the MMA's critical path.
__device__ __forceinline__ void mbar_arrive_relaxed(uint32_t bar) {
    asm volatile("mbarrier.arrive.relaxed.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// One try of a phase wait.  (A suspend-time hint here, and a nanosleep back-off in
// mbar_wait, were both measured: neither changed a conv's time.)
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

// Bounded wait for the phase with the given parity to complete: false after
// `limit` clock cycles without completion.  The clock is read once per 8 tries
// (a try per clock read made the polling warps issue several times more
// instructions than the tries themselves).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, long long limit) {
    if (mbar_try(bar, parity)) return true;
    const long long t0 = clock64();
    while (true) {
#pragma unroll
        for (int k = 0; k < 8; ++k)
            if (mbar_try(bar, parity)) return true;
        if (clock64() - t0 > limit) return false;
    }
}

// The same wait by every lane of a converged warp; the result is made warp-uniform.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, long long limit) {
    const bool ok = mbar_wait(bar, parity, limit);
    return __all_sync(0xffffffffu, ok);
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

// Programmatic dependent launch: the forward's kernels are launched so that the
// next one may start while this one drains.  launch_dependents lets it be
// scheduled; wait blocks until every earlier kernel of the stream has completed
// and its memory is visible -- executed before the first read of anything an
// earlier kernel wrote.  (Both are no-ops without the launch attribute.)
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

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

// One lane of a converged warp (elect.sync) issues the MMA.  The issuing warp
// runs its control loop with all 32 lanes: descriptors and counters stay
// warp-uniform, and the issue keeps its pace while the epilogue warps that
// share its scheduler are busy (a lone issuing lane inside a divergent branch
// issued N=64 MMAs several times slower under that load).
__device__ __forceinline__ void mma_i8_elect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// The KS = CB/32 MMAs of one K chunk (K offsets 0, 32, 64, 96 bytes: descriptor
// start +2 per 32 bytes) in one asm block: one election and one accumulate
// predicate per chunk, one 64-bit add per further MMA.
template <int KS>
__device__ __forceinline__ void mma_chunk_elect(uint32_t d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
    static_assert(KS == 1 || KS == 2 || KS == 4, "K chunk of 32, 64 or 128 bytes");
    if constexpr (KS == 1) {
        asm volatile(
            "{\n\t.reg .pred e, p;\n\t"
            "elect.sync _|e, 0xffffffff;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
            "l"(da), "l"(db), "r"(idesc), "r"(acc)
            : "memory");
    } else if constexpr (KS == 2) {
        asm volatile(
            "{\n\t.reg .pred e, p;\n\t.reg .b64 a1, b1;\n\t"
            "elect.sync _|e, 0xffffffff;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t"
            "add.s64 a1, %1, 2;\n\t"
            "add.s64 b1, %2, 2;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::i8 [%0], a1, b1, %3, 1;\n\t}\n" ::"r"(d),
            "l"(da), "l"(db), "r"(idesc), "r"(acc)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred e, p;\n\t.reg .b64 a1, b1, a2, b2, a3, b3;\n\t"
            "elect.sync _|e, 0xffffffff;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t"
            "add.s64 a1, %1, 2;\n\t"
            "add.s64 b1, %2, 2;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::i8 [%0], a1, b1, %3, 1;\n\t"
            "add.s64 a2, %1, 4;\n\t"
            "add.s64 b2, %2, 4;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::i8 [%0], a2, b2, %3, 1;\n\t"
            "add.s64 a3, %1, 6;\n\t"
            "add.s64 b3, %2, 6;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::i8 [%0], a3, b3, %3, 1;\n\t}\n" ::"r"(d),
            "l"(da), "l"(db), "r"(idesc), "r"(acc)
            : "memory");
    }
}

// All MMAs of one 3x3 halo-block K chunk in one asm block with one election: A
// descriptors of kernel row i start at a0 + i*arow (16-byte units; tap column j and
// K slice k add the immediate j*CB/16 + 2k), B descriptors of tap t at b0 + t*btap
// (+ 2k).  Only the low descriptor word carries the start address (14 bits, never
// carrying into the high word inside shared memory), so each MMA costs two 32-bit
// adds and the tensor-core instruction: issued this way the MMAs run at the tensor
// core's rate (48 cycles per N = 64 MMA, 64 per N = 128), where one asm block per tap
// with 64-bit descriptor arithmetic left the issuing warp at about 70-90 cycles per MMA.
template <int KS>
__device__ __forceinline__ void mma_3x3_chunk(uint32_t d, uint64_t da, uint64_t db, uint32_t arow, uint32_t btap,
                                              uint32_t idesc, uint32_t acc);
template <>
__device__ __forceinline__ void mma_3x3_chunk<1>(uint32_t d, uint64_t da, uint64_t db, uint32_t arow, uint32_t btap,
                                                 uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\t.reg .b32 alo, ahi, blo, bhi, a1, a2, b1, b2, b3, b4, b5, b6, b7, b8, ta, tb;\n\t.reg .b64 A, B;\n\t"
        "mov.b64 {alo, ahi}, %1;\n\tmov.b64 {blo, bhi}, %2;\n\t"
        "add.u32 a1, alo, %5;\n\tadd.u32 a2, a1, %5;\n\t"
        "add.u32 b1, blo, %6;\n\tadd.u32 b2, b1, %6;\n\tadd.u32 b3, b2, %6;\n\tadd.u32 b4, b3, %6;\n\t"
        "add.u32 b5, b4, %6;\n\tadd.u32 b6, b5, %6;\n\tadd.u32 b7, b6, %6;\n\tadd.u32 b8, b7, %6;\n\t"
        "elect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "add.u32 ta, alo, 0;\n\tadd.u32 tb, blo, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, p;\n\t"
        "add.u32 ta, alo, 2;\n\tadd.u32 tb, b1, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, alo, 4;\n\tadd.u32 tb, b2, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a1, 0;\n\tadd.u32 tb, b3, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a1, 2;\n\tadd.u32 tb, b4, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a1, 4;\n\tadd.u32 tb, b5, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a2, 0;\n\tadd.u32 tb, b6, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a2, 2;\n\tadd.u32 tb, b7, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a2, 4;\n\tadd.u32 tb, b8, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "}\n"
        ::"r"(d), "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(arow), "r"(btap)
        : "memory");
}

template <>
__device__ __forceinline__ void mma_3x3_chunk<2>(uint32_t d, uint64_t da, uint64_t db, uint32_t arow, uint32_t btap,
                                                 uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\t.reg .b32 alo, ahi, blo, bhi, a1, a2, b1, b2, b3, b4, b5, b6, b7, b8, ta, tb;\n\t.reg .b64 A, B;\n\t"
        "mov.b64 {alo, ahi}, %1;\n\tmov.b64 {blo, bhi}, %2;\n\t"
        "add.u32 a1, alo, %5;\n\tadd.u32 a2, a1, %5;\n\t"
        "add.u32 b1, blo, %6;\n\tadd.u32 b2, b1, %6;\n\tadd.u32 b3, b2, %6;\n\tadd.u32 b4, b3, %6;\n\t"
        "add.u32 b5, b4, %6;\n\tadd.u32 b6, b5, %6;\n\tadd.u32 b7, b6, %6;\n\tadd.u32 b8, b7, %6;\n\t"
        "elect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "add.u32 ta, alo, 0;\n\tadd.u32 tb, blo, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, p;\n\t"
        "add.u32 ta, alo, 2;\n\tadd.u32 tb, blo, 2;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, alo, 4;\n\tadd.u32 tb, b1, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, alo, 6;\n\tadd.u32 tb, b1, 2;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, alo, 8;\n\tadd.u32 tb, b2, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, alo, 10;\n\tadd.u32 tb, b2, 2;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a1, 0;\n\tadd.u32 tb, b3, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a1, 2;\n\tadd.u32 tb, b3, 2;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a1, 4;\n\tadd.u32 tb, b4, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a1, 6;\n\tadd.u32 tb, b4, 2;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a1, 8;\n\tadd.u32 tb, b5, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a1, 10;\n\tadd.u32 tb, b5, 2;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a2, 0;\n\tadd.u32 tb, b6, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a2, 2;\n\tadd.u32 tb, b6, 2;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a2, 4;\n\tadd.u32 tb, b7, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a2, 6;\n\tadd.u32 tb, b7, 2;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a2, 8;\n\tadd.u32 tb, b8, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a2, 10;\n\tadd.u32 tb, b8, 2;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "}\n"
        ::"r"(d), "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(arow), "r"(btap)
        : "memory");
}

template <>
__device__ __forceinline__ void mma_3x3_chunk<4>(uint32_t d, uint64_t da, uint64_t db, uint32_t arow, uint32_t btap,
                                                 uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\t.reg .b32 alo, ahi, blo, bhi, a1, a2, b1, b2, b3, b4, b5, b6, b7, b8, ta, tb;\n\t.reg .b64 A, B;\n\t"
        "mov.b64 {alo, ahi}, %1;\n\tmov.b64 {blo, bhi}, %2;\n\t"
        "add.u32 a1, alo, %5;\n\tadd.u32 a2, a1, %5;\n\t"
        "add.u32 b1, blo, %6;\n\tadd.u32 b2, b1, %6;\n\tadd.u32 b3, b2, %6;\n\tadd.u32 b4, b3, %6;\n\t"
        "add.u32 b5, b4, %6;\n\tadd.u32 b6, b5, %6;\n\tadd.u32 b7, b6, %6;\n\tadd.u32 b8, b7, %6;\n\t"
        "elect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "add.u32 ta, alo, 0;\n\tadd.u32 tb, blo, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, p;\n\t"
        "add.u32 ta, alo, 2;\n\tadd.u32 tb, blo, 2;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, alo, 4;\n\tadd.u32 tb, blo, 4;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, alo, 6;\n\tadd.u32 tb, blo, 6;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, alo, 8;\n\tadd.u32 tb, b1, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, alo, 10;\n\tadd.u32 tb, b1, 2;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, alo, 12;\n\tadd.u32 tb, b1, 4;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, alo, 14;\n\tadd.u32 tb, b1, 6;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, alo, 16;\n\tadd.u32 tb, b2, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, alo, 18;\n\tadd.u32 tb, b2, 2;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, alo, 20;\n\tadd.u32 tb, b2, 4;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, alo, 22;\n\tadd.u32 tb, b2, 6;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a1, 0;\n\tadd.u32 tb, b3, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a1, 2;\n\tadd.u32 tb, b3, 2;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a1, 4;\n\tadd.u32 tb, b3, 4;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a1, 6;\n\tadd.u32 tb, b3, 6;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a1, 8;\n\tadd.u32 tb, b4, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a1, 10;\n\tadd.u32 tb, b4, 2;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a1, 12;\n\tadd.u32 tb, b4, 4;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a1, 14;\n\tadd.u32 tb, b4, 6;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a1, 16;\n\tadd.u32 tb, b5, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a1, 18;\n\tadd.u32 tb, b5, 2;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a1, 20;\n\tadd.u32 tb, b5, 4;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a1, 22;\n\tadd.u32 tb, b5, 6;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a2, 0;\n\tadd.u32 tb, b6, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a2, 2;\n\tadd.u32 tb, b6, 2;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a2, 4;\n\tadd.u32 tb, b6, 4;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a2, 6;\n\tadd.u32 tb, b6, 6;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a2, 8;\n\tadd.u32 tb, b7, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a2, 10;\n\tadd.u32 tb, b7, 2;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a2, 12;\n\tadd.u32 tb, b7, 4;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a2, 14;\n\tadd.u32 tb, b7, 6;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a2, 16;\n\tadd.u32 tb, b8, 0;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a2, 18;\n\tadd.u32 tb, b8, 2;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a2, 20;\n\tadd.u32 tb, b8, 4;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "add.u32 ta, a2, 22;\n\tadd.u32 tb, b8, 6;\n\t"
        "mov.b64 A, {ta, ahi};\n\tmov.b64 B, {tb, bhi};\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], A, B, %3, 1;\n\t"
        "}\n"
        ::"r"(d), "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(arow), "r"(btap)
        : "memory");
}

__device__ __forceinline__ void mma_commit_elect(uint32_t bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(bar)
        : "memory");
}

// True in exactly one lane of the converged warp.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred;
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, e;\n\t}\n"
        : "=r"(pred));
    return pred != 0;
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
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32"
        " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// The same wait, naming the 16 registers of an earlier tmem_ld16 as read and written, so
// that the compiler keeps every use of them after it (a load whose wait comes later than
// the next instructions, issued ahead of the computation on the previous load).
// Compiler-ordering pins for the software-pipelined TMEM loads (no instruction is
// emitted): pin_after makes the computation on v start after the preceding asm
// statements (the next half's load issue); pin_before makes the values w be computed
// before the following asm statements (the wait for that load).
__device__ __forceinline__ void pin_after(uint32_t (&v)[16]) {
    asm volatile(""
                 : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                   "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]),
                   "+r"(v[15]));
}
__device__ __forceinline__ void pin_before(const uint32_t (&w)[4]) {
    asm volatile("" ::"r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]));
}
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&v)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                   "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]),
                   "+r"(v[15])
                 :
                 : "memory");
}

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

// Four ints -> four saturated int8 in byte order a, b, c, d.
// cvt.pack.sat.s8.s32.b32 d, x, y, z gives {z[15:0], sat(x), sat(y)}.
__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
    uint32_t out;
    asm("{\n\t.reg .b32 t;\n\t"
        "cvt.pack.sat.s8.s32.b32 t, %4, %3, 0;\n\t"
        "cvt.pack.sat.s8.s32.b32 %0, %2, %1, t;\n\t}\n"
        : "=r"(out)
        : "r"(a), "r"(b), "r"(c), "r"(d));
    return out;
}

__device__ __forceinline__ int8_t sat8(int q) { return static_cast<int8_t>(min(max(q, -128), 127)); }

// Exact int8 code (as an int) of one value: the fast estimate unless it is near a tie.
__device__ __forceinline__ int quant_code(float x, float inv, double s);

// 1.5 * 2^23: for |v| < 2^22, v + kRoundMagic lands in [2^23, 2^24) where the
// float spacing is 1, so the addition rounds v to the nearest integer (ties to
// even) and the integer is the low mantissa bits.
constexpr float kRoundMagic = 12582912.0f;
constexpr int kRoundMagicBits = 0x4B400000;

// int32 accumulator -> float, exact for |acc| < 2^22 (then equal to the RNE
// conversion); *flag is raised when acc is outside that range.
__device__ __forceinline__ float acc_to_float(uint32_t acc, uint32_t& flag) {
    flag |= (acc + 0x400000u) >= 0x800000u;
    return __fsub_rn(__int_as_float(static_cast<int>(acc) + kRoundMagicBits), kRoundMagic);
}

// Code estimate of y for scale 1/inv: nearest integer of t = y*inv clamped to
// +-4096 (codes saturate far earlier).  *flag is raised when t lies within
// 1e-4 of a half-integer: there the reference's float64 formula decides.
//
// Only the lower side needs a clamp: for t >= 2^22 the sum's exponent grows and
// the extracted integer is a large positive number that pack4 saturates to
// 127; whenever that happens the tie test also fails, so the exact formula
// confirms it.  Values below -4096 are clamped (codes saturate at -128 long
// before), which keeps the extracted integer from wrapping.
__device__ __forceinline__ int quant_fast(float y, float inv, uint32_t& flag) {
    const float t = fmaxf(__fmul_rn(y, inv), -4096.0f);
    const float m = __fadd_rn(t, kRoundMagic);
    flag |= fabsf(__fsub_rn(t, __fsub_rn(m, kRoundMagic))) >= 0.4999f;
    return __float_as_int(m) - kRoundMagicBits;
}

// Exact reference code of y: clip(round_half_away(double(y) / s), -128, 127).
__device__ __forceinline__ int quant_exact(float y, double s) {
    const double v = static_cast<double>(y) / s;
    double q = v >= 0.0 ? floor(v + 0.5) : ceil(v - 0.5);
    q = fmin(fmax(q, -128.0), 127.0);
    return static_cast<int>(q);
}

// Two-lane float add with one IEEE rounding per lane (add.rn.f32x2).
//
// The dequantization's multiply and add stay scalar (__fmul_rn, __fadd_rn): on
// sm_100a with CUDA 12.9, the packed pair -- written as inline-asm mul.rn.f32x2
// followed by add.rn.f32x2, and again as the __fmul2_rn / __fadd2_rn intrinsics --
// gave codes one step away from the two separate roundings in a few values per
// million, as a fused multiply-add would.
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
    float2 r;
    asm("{\n\t.reg .b64 pa, pb, pd;\n\t"
        "mov.b64 pa, {%2, %3};\n\t"
        "mov.b64 pb, {%4, %5};\n\t"
        "add.rn.f32x2 pd, pa, pb;\n\t"
        "mov.b64 {%0, %1}, pd;\n\t}"
        : "=f"(r.x), "=f"(r.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return r;
}

// Multipliers that bracket 1/s, inv_lo < 1/s < inv_hi (relative gaps near
// 2^-22), and the float32 values y_lo ~ -128 s, y_hi ~ 127 s past which codes
// saturate.  y_hi / s and y_lo / s are within 2^-24 relative of 127 and -128, so
// clamping y to [y_lo, y_hi] never changes a code.
struct QParams {
    float inv_lo, inv_hi, y_lo, y_hi;
};

// Precondition: s finite and positive (callers validate the range first; an infinite
// or NaN scale would leave the bracketing loops below without an exit).
inline bool qparams_scale_ok(double s) { return std::isfinite(s) && s > 0.0; }

inline QParams make_qparams(double s) {
    if (!qparams_scale_ok(s)) return {0.0f, 0.0f, 0.0f, 0.0f};
    const double inv = 1.0 / s;
    float lo = static_cast<float>(inv * (1.0 - 0x1p-22));
    float hi = static_cast<float>(inv * (1.0 + 0x1p-22));
    while (static_cast<double>(lo) >= inv * (1.0 - 0x1p-23)) lo = std::nextafter(lo, 0.0f);
    while (static_cast<double>(hi) <= inv * (1.0 + 0x1p-23)) hi = std::nextafter(hi, HUGE_VALF);
    return {lo, hi, static_cast<float>(-128.0 * s), static_cast<float>(127.0 * s)};
}

// Rare path: 16 codes with the exact formula (kept out of line: small hot loop).
__device__ __noinline__ void quant16_exact(const float* y, double s, uint32_t* w) {
    for (int j = 0; j < 4; ++j)
        w[j] = pack4(quant_exact(y[4 * j], s), quant_exact(y[4 * j + 1], s), quant_exact(y[4 * j + 2], s),
                     quant_exact(y[4 * j + 3], s));
}

// 16 codes clip(round_half_away(double(y[j]) / s), -128, 127) packed into 4 words
// (byte b of word k = code 4k+b).
//
// Each clamped y is multiplied by both bracketing multipliers with 1.5*2^23
// added in the same FMA.  |y * inv| < 2^8, so the exact sum lies in
// [2^23, 2^24) where the float spacing is 1: the FMA returns 1.5*2^23 +
// RNE(y * inv), and the code is the low byte of its bits.  When the two results
// agree on an integer k, the closed interval [y*inv_lo, y*inv_hi] sits inside
// [k-1/2, k+1/2]; double(y)/s lies strictly inside that interval with a gap far
// larger than its float64 rounding, so it rounds (half away) to k as well.
// Otherwise a half-integer lies in between and the float64 formula decides for
// the 16 values.  LOWER: y may lie below y_lo (false when y >= 0 is known).
template <bool LOWER>
__device__ __forceinline__ void quant16q(const float (&y)[16], const QParams& q, double s, uint32_t (&w)[4]) {
    const float2 lo2 = make_float2(q.inv_lo, q.inv_lo);
    const float2 hi2 = make_float2(q.inv_hi, q.inv_hi);
    const float2 mg = make_float2(kRoundMagic, kRoundMagic);
    uint32_t flag = 0, m[16];
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
        float c0 = fminf(y[j], q.y_hi), c1 = fminf(y[j + 1], q.y_hi);
        if (LOWER) {
            c0 = fmaxf(c0, q.y_lo);
            c1 = fmaxf(c1, q.y_lo);
        }
        const float2 c = make_float2(c0, c1);
        const float2 a = __ffma2_rn(c, lo2, mg);
        const float2 b = __ffma2_rn(c, hi2, mg);
        flag |= __float_as_uint(a.x) ^ __float_as_uint(b.x);
        flag |= __float_as_uint(a.y) ^ __float_as_uint(b.y);
        m[j] = __float_as_uint(a.x);
        m[j + 1] = __float_as_uint(a.y);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k)
        w[k] = __byte_perm(__byte_perm(m[4 * k], m[4 * k + 1], 0x0040), __byte_perm(m[4 * k + 2], m[4 * k + 3], 0x0040),
                           0x5410);
    if (flag) {
        // the same clamp first: it may carry a folded activation (fold_act)
        float ys[16];
        uint32_t ws[4];
#pragma unroll
        for (int j = 0; j < 16; ++j) ys[j] = LOWER ? fmaxf(fminf(y[j], q.y_hi), q.y_lo) : fminf(y[j], q.y_hi);
        quant16_exact(ys, s, ws);
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = ws[j];
    }
}

// QParams whose clamp also applies the activation of a conv whose fp32 values are
// not kept: relu then clip to [y_lo, y_hi] is clip(y, 0, y_hi), relu6 is
// clip(y, 0, min(6, y_hi)) (y_lo < 0 < y_hi), so the codes are unchanged.
__device__ __forceinline__ QParams fold_act(QParams q, int act) {
    if (act != 0) q.y_lo = 0.0f;
    if (act == 2) q.y_hi = fminf(q.y_hi, 6.0f);
    return q;
}

__device__ __forceinline__ int quant_code(float x, float inv, double s) {
    uint32_t flag = 0;
    const int q = quant_fast(x, inv, flag);
    return flag ? quant_exact(x, s) : q;
}

// Global loads and stores of the epilogues and producers: activations are read once and
// written once, so they bypass L1 (.L1::no_allocate).  Letting the epilogue's stores
// allocate L1 lines made the dense convs of a ResNet-18 forward ~7 % slower in total.
__device__ __forceinline__ void ld_v8(const float* p, float* v) {
    asm volatile("ld.global.nc.L1::no_allocate.v8.f32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7])
                 : "l"(p));
}
__device__ __forceinline__ void st_v8(float* p, const float* v) {
    asm volatile("st.global.L1::no_allocate.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "f"(v[0]), "f"(v[1]),
                 "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
                 : "memory");
}
__device__ __forceinline__ void st_v8(uint32_t* p, const uint32_t* v) {
    asm volatile("st.global.L1::no_allocate.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(v[0]), "r"(v[1]),
                 "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}

__device__ __forceinline__ void st_v4(void* p, uint4 v) {
    asm volatile("st.global.L1::no_allocate.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ void st_u32(void* p, uint32_t v) {
    asm volatile("st.global.L1::no_allocate.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ float apply_act(float y, int act) {
    if (act == 1) return fmaxf(y, 0.0f);
    if (act == 2) return fminf(fmaxf(y, 0.0f), 6.0f);
    return y;
}

// ------------------------------------------------------------------ epilogue outputs

// Layouts: fp32 activations are NHWC [N][H][W][cout]; int8 code tensors are
// NHWC with a one-pixel zero border, [N][H+2][W+2][ldq], so that stride-1
// convs read every tap of a tile from one contiguous block (see conv_tc_kernel).
// fp32 activation maps.  With C % 8 == 0 they are tiled as blocks of 32
// positions x groups of 8 channels: element (p, c) at
// ((p/32) * (C/8) + c/8) * 256 + (p%32) * 8 + c%8.  A thread's 8 channels stay
// one 32-byte row, and the 32 lanes of a warp (consecutive positions) cover
// 1 KB of consecutive bytes.  Other channel counts use plain NHWC [P][C].
// Buffers hold a whole number of 32-position blocks.
__host__ __device__ __forceinline__ size_t f32_off(size_t p, int c, int C) {
    if ((C & 7) == 0)
        return (((p >> 5) * static_cast<size_t>(C >> 3) + static_cast<size_t>(c >> 3)) << 8) + ((p & 31) << 3) +
               static_cast<size_t>(c & 7);
    return p * static_cast<size_t>(C) + c;
}

struct EpiParams {
    const float* factor;    // [cout] float(float(s_in) * w_scale[c])
    const float* bias;      // [cout]
    const float* residual;  // fp32 map [P][cout] (f32_off layout) or null
    float* out_f32;         // fp32 map [P][cout] (f32_off layout) or null
    int8_t* out_q0;         // bordered int8 codes [N][OH+2][OW+2][ldq0] or null
    int8_t* out_q1;
    int ldq0, ldq1;
    float inv0, inv1;
    double s0, s1;
    QParams q0, q1;         // bracketing multipliers / saturation bounds of s0, s1
    int cout;
    int vec32;  // 1 when cout % 8 == 0: tiled fp32 maps, 256-bit loads/stores of 8 channels
    int act;    // activation of the conv itself: 0 none / 1 relu / 2 relu6
    int aux_act;   // AUX: activation of the recomputed residual (its constants are in ConvConsts)
    // bit o set: code output o is written only at even (h, w), into a bordered
    // (sub_h+2) x (sub_w+2) map at (h/2, w/2) -- the input of a fused 1x1 stride-2 conv
    int sub_mask;
    int sub_h, sub_w;
    int acc_small; // 1 when 128 * sum_k |w[c][k]| < 2^22 for every c: no range check in the float conversion
    int post;   // residual: 0 none, 1 add then relu, 2 add only
    // positional decomposition: channel c' = pos*dcr_oc + c of a 1x1 GEMM output is code
    // (pos / dcr_w, pos % dcr_w, c) of a dcr_h x dcr_w map (DepthToSpace, DCR order)
    int dcr_oc, dcr_h, dcr_w;
};

// Element (pf, c) of the conv's output in its fp32 map: the position, channel
// and channel count to pass to f32_off.  A positionally decomposed conv (one
// output position per image, channel c = pos*dcr_oc + c') writes position pos
// of its dcr_h x dcr_w map instead.  c must be the first of a group of 16.
struct F32At {
    size_t p;
    int c, C;
};
__device__ __forceinline__ F32At f32_at(const EpiParams& e, size_t pf, int c) {
    if (e.dcr_oc) {
        const int pos = c / e.dcr_oc;
        return {pf * static_cast<size_t>(e.dcr_h * e.dcr_w) + pos, c - pos * e.dcr_oc, e.dcr_oc};
    }
    return {pf, c, e.cout};
}

// Per-channel dequantization constants of one tensor-core conv, passed as a
// __grid_constant__ kernel parameter: the epilogue reads them through the
// constant cache with warp-uniform addresses.  (Kept in shared memory, these
// broadcast reads took over 40% of the shared-memory pipe that feeds the tensor
// core and slowed the MMAs of the 64-channel convs by a third.)
constexpr int kMaxConstCh = 1536;   // output channels of one conv
constexpr int kMaxAuxCh = 256;      // output channels of an aux GEMM
struct ConvConsts {
    float2 fb[kMaxConstCh];         // (factor, bias) of channel c: one 64-bit load;
                                    // factor = float(float(s_in) * w_scale[c]); zero past cout
    float2 aux_fb[kMaxAuxCh];       // AUX: the recomputed residual's constants
};

// Residual of 16 consecutive channels [c0, c0+16) of fp32 row pf (nv valid).
__device__ __forceinline__ void load_res16(const EpiParams& e, size_t pf, int c0, int nv, float (&r)[16]) {
    const F32At a = f32_at(e, pf, c0);
    if (nv == 16 && e.vec32) {
        ld_v8(e.residual + f32_off(a.p, a.c, a.C), &r[0]);
        ld_v8(e.residual + f32_off(a.p, a.c + 8, a.C), &r[8]);
    } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) r[j] = j < nv ? e.residual[f32_off(a.p, a.c + j, a.C)] : 0.0f;
    }
}

// Dequantize 16 accumulators of channels [c, c+16) (factor/bias: 16 constants
// each, from the kernel parameters): y = act(fadd(fmul(float(acc), factor), bias)),
// two roundings.
//
// float(acc): acc + 0x4B400000 is the bit pattern of 1.5*2^23 + acc when
// |acc| < 2^22 (exact subtraction afterwards); in that range the pattern xor
// 0x4B000000 stays below 2^23, so one OR over the 16 patterns tells whether
// every accumulator was in range.  Otherwise the rounding conversion is used.
// `check` false: the caller knows |acc| < 2^22 (128 * sum |w| < 2^22 for every channel).
// BIASED: v already holds acc + 0x4B400000 (an accumulator that started at the bias;
// the caller knows |acc| < 2^22, `check` is ignored).
template <bool BIASED = false>
__device__ __forceinline__ void dequant16(const uint32_t (&v)[16], const float2* fb, int act, float (&y)[16],
                                          bool check = true) {
    uint32_t range = 0;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const uint32_t bits = BIASED ? v[j] : v[j] + static_cast<uint32_t>(kRoundMagicBits);
        if (check && !BIASED) range |= bits ^ 0x4B000000u;
        y[j] = __uint_as_float(bits);
    }
    if (range < 0x800000u) {
        const float2 mg = make_float2(-kRoundMagic, -kRoundMagic);
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
            const float2 t = add2_rn(make_float2(y[j], y[j + 1]), mg);
            y[j] = t.x;
            y[j + 1] = t.y;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) y[j] = __int2float_rn(static_cast<int>(v[j]));
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const float2 c = fb[j];
        y[j] = __fadd_rn(__fmul_rn(y[j], c.x), c.y);
    }
    if (act == 1) {
#pragma unroll
        for (int j = 0; j < 16; ++j) y[j] = fmaxf(y[j], 0.0f);
    } else if (act == 2) {
#pragma unroll
        for (int j = 0; j < 16; ++j) y[j] = fminf(fmaxf(y[j], 0.0f), 6.0f);
    }
}

// Residual add + post activation and the fp32 store of 16 channels [c0, c0+16) (nv valid).
// POST_RELU false: the caller folds the post-add ReLU into the quantizer's clamp
// (no fp32 values are stored).
template <bool RES, bool F32, bool POST_RELU = true>
__device__ __forceinline__ void finish16(const EpiParams& e, size_t pf, int c0, int nv, float (&y)[16],
                                         const float (&r)[16]) {
    if constexpr (RES) {
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
            const float2 t = add2_rn(make_float2(y[j], y[j + 1]), make_float2(r[j], r[j + 1]));
            y[j] = t.x;
            y[j + 1] = t.y;
        }
        if (POST_RELU && e.post == 1) {
#pragma unroll
            for (int j = 0; j < 16; ++j) y[j] = fmaxf(y[j], 0.0f);
        }
    }
    if constexpr (F32) {
        const F32At a = f32_at(e, pf, c0);
        if (nv == 16 && e.vec32) {
            st_v8(e.out_f32 + f32_off(a.p, a.c, a.C), &y[0]);
            st_v8(e.out_f32 + f32_off(a.p, a.c + 8, a.C), &y[8]);
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (j < nv) e.out_f32[f32_off(a.p, a.c + j, a.C)] = y[j];
        }
    }
}

// Whether output o keeps the code of position (h, w) (subsampled outputs keep even positions).
__device__ __forceinline__ bool code_kept(const EpiParams& e, int o, int h, int w) {
    return !((e.sub_mask >> o) & 1) || ((h | w) & 1) == 0;
}

// Code row of output o for channel c0 (bordered layout; positional decomposition remaps;
// subsampled outputs address the half-size map).
__device__ __forceinline__ int8_t* code_ptr(const EpiParams& e, int o, size_t pq, int n, int c0, int h, int w) {
    int cq = c0;
    if ((e.sub_mask >> o) & 1) {
        pq = (static_cast<size_t>(n) * (e.sub_h + 2) + (h >> 1) + 1) * (e.sub_w + 2) + (w >> 1) + 1;
    } else if (e.dcr_oc) {
        const int pos = c0 / e.dcr_oc;
        cq = c0 - pos * e.dcr_oc;
        pq = (static_cast<size_t>(n) * (e.dcr_h + 2) + pos / e.dcr_w + 1) * (e.dcr_w + 2) + pos % e.dcr_w + 1;
    }
    return (o == 0 ? e.out_q0 : e.out_q1) + pq * static_cast<size_t>(o == 0 ? e.ldq0 : e.ldq1) + cq;
}

// ------------------------------------------------------------------ tensor-core conv

// Division of 32-bit unsigned values by a fixed divisor d as one multiply-high:
// with m = ceil(2^64 / d), x*m/2^64 = x/d + x*e/(d*2^64) for e = m*d - 2^64 < d,
// and x*e/(d*2^64) < 2^-32 < 1/d, so the floor is exactly floor(x/d) for every
// x < 2^32 (d = 1 is passed through).
struct FastDiv {
    unsigned long long m;
    uint32_t d;
};
inline FastDiv make_fastdiv(uint32_t d) {
    return {d <= 1 ? 0ull : (~0ull) / d + 1ull, d};
}
__device__ __forceinline__ uint32_t fdiv(uint32_t x, const FastDiv& f) {
    return f.d == 1 ? x : static_cast<uint32_t>(__umul64hi(static_cast<unsigned long long>(x), f.m));
}

struct ConvGeom {
    int mode;                   // 0: per-tap 4-D tile loads; 1: one halo block per tile, taps = shifted views;
                                // 2: stride-2 3x3 over 64-byte pixels, one 4-D box of pixel pairs per two taps
    int N, OH, OW;              // output map (per image)
    // mode 0
    int TW, TH, TN;             // one M tile = TN images x TH rows x TW cols (<= 128 positions)
    int tiles_w, tiles_h;       // M tiles along W and H
    int KW, SH, SW, PH, PW;     // kernel width, strides, paddings
    int coord_off;              // 1 when the A tensor carries the one-pixel border
    // positional sub-convs (mode 0, TW = TH = 1): a tile is one output position of TN
    // images, and only the taps that read inside the IH x IW input are loaded and
    // multiplied (the others would multiply padding code 0)
    int pos_tiles, IH, IW;
    // mode 1 (stride 1, same-size output): tiles are 128 consecutive bordered positions
    int KH, Hp, Wp;             // kernel height, bordered map dims
    int blk_off;                // first block row relative to the tile's first row
    int a_stage;                // bytes per A stage (1024-aligned)
    int m_tiles;                // total M tiles
    int n_cchunks, n_kchunks;   // channel chunks per tap, total K chunks
    int BN;                     // N tile (multiple of 16, <= 256)
    int acc_cols;               // TMEM columns per accumulator buffer (power of two >= max(32, BN))
    int n_acc;                  // accumulator buffers (2, 4 or 8): tiles in flight between MMA and epilogue
    int n_groups;               // epilogue warp groups (2 or 4); group gi drains buffers gi, gi + n_groups, ...
    int stages;                 // A (and streamed B) pipeline depth, <= kMaxStages
    int b_resident;             // 1: the CTA's whole weight slab stays in shared memory
    uint32_t a_bytes, b_bytes;  // TMA bytes per A stage / per B chunk
    // aux GEMM (AUX kernels): a second 1x1 GEMM with K = aux_kb (32, 64 or 128)
    // bytes per row, over rows aligned with the tile's rows, into a second
    // accumulator; its dequantized output is the residual (a block identity
    // recomputed instead of stored in fp32)
    int aux_off;                // byte offset of the aux A tile (128 rows x aux_kb bytes) inside each A stage
    uint32_t aux_bytes;         // TMA bytes of that tile
    int aux_kb;                 // K bytes of the aux GEMM (its swizzle width)
    int aux_col;                // TMEM column of the aux accumulator inside a buffer
    // divisors of the per-tile position decode
    FastDiv fd_img;             // mode 1: Hp * Wp
    FastDiv fd_wp;              // mode 1: Wp
    FastDiv fd_tiles_w;         // mode 0: tiles along W
    FastDiv fd_tiles_h;         // mode 0: tiles along H
    // failure detection: the engine's device error word (a CTA that finds it set at start
    // skips its work), the bounded-wait limit in clock cycles, and a test switch that makes
    // the first A load of CTA (0, 0) never arrive (its expect_tx is posted, the copy is not
    // issued), so the waits on that stage run out and report instead of hanging
    int* err;
    long long wait_limit;
    int stall_first_load;
    // W4 weights stored two codes per byte (b_packed, resident slabs only): w4 = [w_rows][w4_ld]
    // bytes, byte k/2 of row n holds code k in its low nibble and code k+1 in its high nibble
    // (k even, K-major like the int8 matrix); the epilogue warps unpack the N tile's slab
    // into the swizzled shared-memory layout of the TMA-loaded int8 weights
    const uint8_t* w4;
    int w4_ld, w_rows, b_packed;
};

// Kernel rows [kh0, kh1) and columns [kw0, kw1) that M tile mt multiplies: all of them,
// or (positional sub-convs) those of its output position that read inside the input.
__device__ __forceinline__ void tile_taps(const ConvGeom& g, int mt, int& kh0, int& kh1, int& kw0, int& kw1) {
    kh0 = 0;
    kh1 = g.KH;
    kw0 = 0;
    kw1 = g.KW;
    if (g.pos_tiles) {
        const uint32_t rest = fdiv(static_cast<uint32_t>(mt), g.fd_tiles_w);
        const uint32_t nb = fdiv(rest, g.fd_tiles_h);
        const int ow = static_cast<int>(static_cast<uint32_t>(mt) - rest * g.fd_tiles_w.d);
        const int oh = static_cast<int>(rest - nb * g.fd_tiles_h.d);
        const int ih = oh * g.SH - g.PH, iw = ow * g.SW - g.PW;   // input row / column of kernel tap 0
        kh0 = max(0, -ih);
        kh1 = min(g.KH, g.IH - ih);
        kw0 = max(0, -iw);
        kw1 = min(g.KW, g.IW - iw);
    }
}

// Sign-extended int8 codes of the 8 int4 codes in packed word x (low nibble first):
// lo/hi = codes 8i+0..3 / 8i+4..7 as bytes.
__device__ __forceinline__ void unpack_w4(uint32_t x, uint32_t& lo, uint32_t& hi) {
    uint32_t a = x & 0x0F0F0F0Fu;          // codes 0, 2, 4, 6 (nibbles)
    uint32_t b = (x >> 4) & 0x0F0F0F0Fu;   // codes 1, 3, 5, 7
    a |= (a & 0x08080808u) * 0x1Eu;        // nibble bit 3 set -> byte 0xF0 | nibble (no carry between bytes)
    b |= (b & 0x08080808u) * 0x1Eu;
    lo = __byte_perm(a, b, 0x5140);        // a.b0 b.b0 a.b1 b.b1
    hi = __byte_perm(a, b, 0x7362);        // a.b2 b.b2 a.b3 b.b3
}

// Make this thread's generic-proxy shared-memory writes visible to the tensor core
// (async proxy) once the consumer has synchronised with it.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

constexpr int kEpiWarps = 16;                      // 4 per TMEM lane quadrant
constexpr int kConvThreads = 64 + 32 * kEpiWarps;  // warp 0 TMA, warp 1 MMA, warps 2.. epilogue
constexpr int kMaxStages = 24;

// Epilogue of a halo-block conv (mode 1) whose single N tile is the whole output:
// cout == FBN (64 or 128, a compile-time constant), no positional decomposition.
// Every channel offset is then a compile-time constant: the (factor, bias) pairs
// are constant-bank operands of the multiply and the add (no loads), the fp32
// row and code-row offsets of a 16-channel half are immediates, and the column
// loop is unrolled.  A thread's row walks the tiles of its group by a fixed step
// of bordered positions, so (image, row, column) advance by carries instead of
// divisions.  Warps: NG groups (4, or 2 when two accumulators fit) of 16 / NG
// warps; group gi drains accumulators gi, gi + NG, ...; with NG = 2 the two warps
// of a lane quadrant split the columns in halves.  Numerics are those of the
// general epilogue below (same dequant16 / quant16q calls in the same order).
template <int CB, int NOUT, bool RES, bool F32, bool AUX, int FBN>
__device__ __forceinline__ void epilogue_fast(const ConvGeom& g, const EpiParams& e, const ConvConsts& cc,
                                              uint32_t tmem, uint32_t accf0, uint32_t acce0, int warp, int lane) {
    static_assert(FBN == 64 || FBN == 128, "fast epilogue: 64 or 128 output channels");
    constexpr int HALVES = FBN / 16;
    const int NG = g.n_groups;
    const int NA = g.n_acc;
    const int gw = kEpiWarps / NG;
    const int ew = warp - 2;
    const int gi = ew / gw;
    const int quad = warp & 3;
    const int slice = (ew % gw) >> 2;
    const int r = quad * 32 + lane;
    const int h_lo = NG == 4 ? 0 : slice * (HALVES / 2);
    const int h_hi = NG == 4 ? HALVES : h_lo + HALVES / 2;
    // quantizer clamps with the activation / post-add ReLU folded where no fp32 value is kept
    constexpr bool kFold = !RES && !F32 && !AUX;
    constexpr bool kFoldPost = RES && !F32;
    const bool nonneg = RES ? e.post == 1 : e.act != 0;
    QParams qx[2] = {e.q0, e.q1};
    if (kFold) {
        qx[0] = fold_act(e.q0, e.act);
        qx[1] = fold_act(e.q1, e.act);
    } else if (nonneg) {
        qx[0].y_lo = 0.0f;
        qx[1].y_lo = 0.0f;
    }
    const double sq[2] = {e.s0, e.s1};
    const int act = kFold ? 0 : e.act;
    const bool check = !e.acc_small;
    griddep_wait();   // residuals are earlier kernels' outputs

    const uint32_t img = g.fd_img.d, Wp = g.fd_wp.d, Hp = static_cast<uint32_t>(g.Hp);
    const uint32_t step = static_cast<uint32_t>(NG) * gridDim.x * 128u;
    uint32_t q = (blockIdx.x + static_cast<uint32_t>(gi) * gridDim.x) * 128u + static_cast<uint32_t>(r);
    uint32_t n = fdiv(q, g.fd_img);
    uint32_t hb = fdiv(q - n * img, g.fd_wp);
    uint32_t wb = q - n * img - hb * Wp;
    const uint32_t sn = fdiv(step, g.fd_img);
    const uint32_t sh = fdiv(step - sn * img, g.fd_wp);
    const uint32_t sw = step - sn * img - sh * Wp;

    int buf = gi;
    uint32_t use = 0;
    for (int mt = blockIdx.x + gi * gridDim.x; mt < g.m_tiles; mt += NG * gridDim.x) {
        const int h = static_cast<int>(hb) - 1, w = static_cast<int>(wb) - 1;
        const bool valid = n < static_cast<uint32_t>(g.N) && h >= 0 && h < g.OH && w >= 0 && w < g.OW;
        const bool even = ((h | w) & 1) == 0;
        // fp32 map offset of channel 0 of this position (tiled layout, C = FBN)
        const uint32_t pf = (n * static_cast<uint32_t>(g.OH) + static_cast<uint32_t>(h)) * static_cast<uint32_t>(g.OW) +
                            static_cast<uint32_t>(w);
        const size_t fo = static_cast<size_t>(pf >> 5) * (FBN * 32) + (pf & 31u) * 8u;
        int8_t* qrow[2] = {nullptr, nullptr};
        bool kept[2] = {false, false};
#pragma unroll
        for (int o = 0; o < NOUT; ++o) {
            const bool sub = (e.sub_mask >> o) & 1;
            kept[o] = valid && (!sub || even);
            const size_t pq = sub ? (static_cast<size_t>(n) * (e.sub_h + 2) + (h >> 1) + 1) * (e.sub_w + 2) + (w >> 1) + 1
                                  : static_cast<size_t>(q);
            qrow[o] = (o == 0 ? e.out_q0 : e.out_q1) + pq * static_cast<size_t>(o == 0 ? e.ldq0 : e.ldq1);
        }
        // the residual does not depend on the MMAs: fetch the first half before waiting
        float res[16];
        if (RES && !AUX && valid) {
            ld_v8(e.residual + fo + static_cast<size_t>(2 * h_lo) * 256, &res[0]);
            ld_v8(e.residual + fo + static_cast<size_t>(2 * h_lo + 1) * 256, &res[8]);
        }
        if (!mbar_wait(accf0 + 8 * buf, use & 1u, g.wait_limit)) {
            atomicExch(g.err, ERR_WAIT_ACC);
            break;
        }
        tc_fence_after();
        const uint32_t trow = tmem + static_cast<uint32_t>(buf * g.acc_cols) + (static_cast<uint32_t>(quad * 32) << 16);
        uint32_t wq[2][8];
        // accumulators of half hh in v[hh & 1] (h_lo is even).  Without a residual the load of
        // the next half is issued before this half's arithmetic and waited for after it, so its
        // TMEM latency overlaps the computation; with one, each half is loaded and waited for in
        // turn (the second buffer pushed the residual kernels into spills: layer1.1.conv2 0.886 ms
        // pipelined against 0.839 ms without)
        uint32_t v[2][16], vx[2][16];
        constexpr bool kPipe = !RES;
        if (kPipe) {
            __syncwarp();   // each lane left the accumulator wait on its own
            tmem_ld16(trow + h_lo * 16, v[0]);
            if (AUX) tmem_ld16(trow + static_cast<uint32_t>(g.aux_col) + h_lo * 16, vx[0]);
            tmem_wait_ld(v[0]);
            if (AUX) tmem_wait_ld(vx[0]);
        }
#pragma unroll
        for (int hh = 0; hh < HALVES; ++hh) {
            if (hh < h_lo || hh >= h_hi) continue;
            const int cur = hh & 1, nxt = cur ^ 1;
            __syncwarp();   // tcgen05.ld is .sync.aligned: reconverge after the per-lane stores
            if (!kPipe) {
                tmem_ld16(trow + hh * 16, v[cur]);
                if (AUX) tmem_ld16(trow + static_cast<uint32_t>(g.aux_col) + hh * 16, vx[cur]);
                tmem_wait_ld(v[cur]);
                if (AUX) tmem_wait_ld(vx[cur]);
            } else if (hh + 1 < h_hi) {
                tmem_ld16(trow + (hh + 1) * 16, v[nxt]);
                if (AUX) tmem_ld16(trow + static_cast<uint32_t>(g.aux_col) + (hh + 1) * 16, vx[nxt]);
                pin_after(v[cur]);
                if (AUX) pin_after(vx[cur]);
            }
            if (valid) {
            float y[16];
            dequant16(v[cur], cc.fb + hh * 16, act, y, check);
            if (AUX) dequant16(vx[cur], cc.aux_fb + hh * 16, e.aux_act, res, false);   // aux K <= 128
            if constexpr (RES) {
#pragma unroll
                for (int j = 0; j < 16; j += 2) {
                    const float2 t = add2_rn(make_float2(y[j], y[j + 1]), make_float2(res[j], res[j + 1]));
                    y[j] = t.x;
                    y[j + 1] = t.y;
                }
                if (!kFoldPost && e.post == 1) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) y[j] = fmaxf(y[j], 0.0f);
                }
            }
            if constexpr (F32) {
                st_v8(e.out_f32 + fo + static_cast<size_t>(2 * hh) * 256, &y[0]);
                st_v8(e.out_f32 + fo + static_cast<size_t>(2 * hh + 1) * 256, &y[8]);
            }
            if (RES && !AUX && hh + 1 < h_hi) {   // next half's residual
                ld_v8(e.residual + fo + static_cast<size_t>(2 * hh + 2) * 256, &res[0]);
                ld_v8(e.residual + fo + static_cast<size_t>(2 * hh + 3) * 256, &res[8]);
            }
#pragma unroll
            for (int o = 0; o < NOUT; ++o) {
                if (!kept[o]) continue;
                uint32_t w4[4];
                quant16q<true>(y, qx[o], sq[o], w4);
                pin_before(w4);
#pragma unroll
                for (int j = 0; j < 4; ++j) wq[o][(hh & 1) * 4 + j] = w4[j];
                if (hh & 1) st_v8(reinterpret_cast<uint32_t*>(qrow[o] + (hh >> 1) * 32), wq[o]);
            }
            }
            if (kPipe && hh + 1 < h_hi) {
                __syncwarp();
                tmem_wait_ld(v[nxt]);
                if (AUX) tmem_wait_ld(vx[nxt]);
            }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_relaxed(acce0 + 8 * buf);
        if ((buf += NG) >= NA) {
            buf -= NA;
            use ^= 1u;
        }
        // next tile of this group: step bordered positions further
        wb += sw;
        if (wb >= Wp) {
            wb -= Wp;
            ++hb;
        }
        hb += sh;
        if (hb >= Hp) {
            hb -= Hp;
            ++n;
        }
        n += sn;
        q += step;
    }
}

// Persistent implicit-GEMM conv.  grid = (CTAs per N tile, N tiles); each CTA
// walks M tiles blockIdx.x, blockIdx.x + gridDim.x, ...  Two TMEM accumulators
// let the epilogue of tile i overlap the MMAs of tile i+1.
//
// mode 0: every K chunk (tap, channel chunk) is its own 4-D TMA box of the
//         input (element strides give stride 2; out-of-range boxes read zeros).
// mode 1: a tile is 128 consecutive positions of the bordered map; one 2-D box
//         of 128 + (KH-1)*Wp + KW-1 bordered rows per channel chunk holds every
//         tap, and tap (i, j) is the same shared-memory block seen from row
//         i*Wp + j.  Border outputs are computed and dropped.
// Template parameters fix the per-launch shape of the work so each launch runs
// a lean instruction stream: CB = K-chunk bytes (swizzle width), MODE (above),
// NOUT = int8 code outputs (0..2), RES = residual add, F32 = fp32 output,
// AUX = the residual is the aux GEMM's output (map_xa / map_xb) instead of a load,
// FBN = 64 / 128: mode 1 with that whole-output N tile, drained by epilogue_fast.
template <int CB, int MODE, int NOUT, bool RES, bool F32, bool AUX, int FBN = 0>
__global__ void __launch_bounds__(kConvThreads, 1)
conv_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
               const __grid_constant__ CUtensorMap map_xa, const __grid_constant__ CUtensorMap map_xb,
               const ConvGeom g, const EpiParams e, const __grid_constant__ ConvConsts cc) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ int s_abort;
    __shared__ __align__(8) uint64_t bars[2 * kMaxStages + 18];  // a_full, a_empty, b_full, acc_full[8], acc_empty[8], done
    __shared__ uint32_t tslot;
    // A wait of an earlier CTA already ran out: skip the work (block-uniform decision).
    if (threadIdx.x == 0) s_abort = *reinterpret_cast<volatile int*>(g.err);
    __syncthreads();
    if (s_abort) return;

    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int BN = g.BN;
    const int bn32 = (BN + 31) & ~31;
    const int S = g.stages;
    const int sb_stride = (BN * CB + 1023) & ~1023;   // every B chunk 1024-byte aligned (swizzle atoms)
    uint8_t* sA = smem;
    uint8_t* sB = smem + S * g.a_stage;
    uint8_t* sBx = sB + (g.b_resident ? g.n_kchunks : S) * sb_stride;   // aux weights [BN][aux_kb] (AUX)

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nt = blockIdx.y;
    const uint32_t full0 = smem_u32(&bars[0]);
    const uint32_t empty0 = smem_u32(&bars[kMaxStages]);
    const uint32_t bfull = smem_u32(&bars[2 * kMaxStages]);
    const uint32_t accf0 = smem_u32(&bars[2 * kMaxStages + 1]);
    const uint32_t acce0 = smem_u32(&bars[2 * kMaxStages + 9]);
    const uint32_t donebar = smem_u32(&bars[2 * kMaxStages + 17]);
    const int NA = g.n_acc;
    const int NG = g.n_groups;
    const int group_warps = kEpiWarps / NG;   // epilogue warps per group (multiple of 4)

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        // resident weights: the producer's TMA loads (int8 slab, or the aux weights only when
        // the slab is packed) and, for a packed slab, the epilogue warps' unpack
        mbar_init(bfull, (g.b_packed ? 1u : 0u) + ((!g.b_packed || AUX) ? 1u : 0u));
        for (int b = 0; b < NA; ++b) {
            mbar_init(accf0 + 8 * b, 1);
            mbar_init(acce0 + 8 * b, group_warps);
        }
        mbar_init(donebar, 1);
        fence_mbar_init();
        tma_prefetch(&map_a);
        tma_prefetch(&map_b);
        if (AUX) {
            tma_prefetch(&map_xa);
            tma_prefetch(&map_xb);
        }
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&tslot), NA * g.acc_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    griddep_launch();
    const uint32_t tmem = tslot;
    // A loads per tile (mode 2: a pair box and a single-tap box per kernel row)
    const int n_a = MODE == 1 ? g.n_cchunks : (MODE == 2 ? 2 * g.KH : g.n_kchunks);

    if (warp == 0) {
        // ---------------- TMA producer (whole warp; one elected lane issues the copies)
        uint32_t last_ph = 0;   // bit s: parity of the last load issued into stage s
        uint32_t used = 0;      // bit s: stage s received at least one load
        bool ok = true;
        if (g.b_resident && (!g.b_packed || AUX)) {
            if (elect_one()) {
                mbar_expect_tx(bfull, (g.b_packed ? 0u : g.b_bytes * g.n_kchunks) +
                                          (AUX ? static_cast<uint32_t>(BN * g.aux_kb) : 0u));
                if (!g.b_packed)
                    for (int kc = 0; kc < g.n_kchunks; ++kc)
                        tma_load_2d(smem_u32(sB + kc * sb_stride), &map_b, bfull, kc * CB, nt * BN);
                if (AUX) tma_load_2d(smem_u32(sBx), &map_xb, bfull, 0, nt * BN);
            }
            __syncwarp();
        }
        int s = 0;
        uint32_t ph = 0;
        griddep_wait();   // A tiles (and the aux rows) are earlier kernels' outputs
        for (int mt = blockIdx.x; ok && mt < g.m_tiles; mt += gridDim.x) {
            int w0 = 0, h0 = 0, n0 = 0;
            if (MODE == 0 || MODE == 2) {
                const uint32_t rest = fdiv(static_cast<uint32_t>(mt), g.fd_tiles_w);
                const uint32_t nb = fdiv(rest, g.fd_tiles_h);
                w0 = static_cast<int>(static_cast<uint32_t>(mt) - rest * g.fd_tiles_w.d) * g.TW;
                h0 = static_cast<int>(rest - nb * g.fd_tiles_h.d) * g.TH;
                n0 = static_cast<int>(nb) * g.TN;
            }
            int kh0 = 0, kh1 = 1, kw0 = 0, kw1 = 1;
            if (MODE == 0) tile_taps(g, mt, kh0, kh1, kw0, kw1);
            const int na = MODE == 0 ? (kh1 - kh0) * (kw1 - kw0) * g.n_cchunks : n_a;
            int ki = kh0, kj = kw0, cc = 0;
            for (int ka = 0; ka < na; ++ka) {
                if (!mbar_wait_warp(empty0 + 8 * s, ph ^ 1, g.wait_limit)) {
                    if (lane == 0) atomicExch(g.err, ERR_WAIT_EMPTY);
                    ok = false;
                    break;
                }
                const uint32_t fb = full0 + 8 * s;
                // test switch: the bytes of this stage are announced but never copied
                const bool stall = g.stall_first_load && ka == 0 && mt == 0 && blockIdx.y == 0;
                if (elect_one()) {
                    const bool aux = AUX && ka == 0;
                    mbar_expect_tx(fb, g.a_bytes + (g.b_resident ? 0u : g.b_bytes) + (aux ? g.aux_bytes : 0u));
                }
                if (!stall && elect_one()) {
                    const bool aux = AUX && ka == 0;
                    if (aux) tma_load_2d(smem_u32(sA + s * g.a_stage + g.aux_off), &map_xa, fb, 0, mt * 128);
                    if (MODE == 1) {
                        tma_load_2d(smem_u32(sA + s * g.a_stage), &map_a, fb, ka * CB, mt * 128 + g.blk_off);
                    } else if (MODE == 2) {
                        // kernel row ka / 2: the pixel pairs (2w, 2w+1) of bordered columns 2w, 2w+1 (taps
                        // 0 and 1) for ka even, the pairs one further (tap 2 in their first half) for ka odd;
                        // bordered input row 2h + kernel row (element stride 2)
                        tma_load_4d(smem_u32(sA + s * g.a_stage), &map_a, fb, 0, w0 + (ka & 1), h0 * 2 + (ka >> 1), n0);
                    } else {
                        tma_load_4d(smem_u32(sA + s * g.a_stage), &map_a, fb, cc * CB,
                                    w0 * g.SW + kj - g.PW + g.coord_off, h0 * g.SH + ki - g.PH + g.coord_off, n0);
                        if (!g.b_resident)
                            tma_load_2d(smem_u32(sB + s * sb_stride), &map_b, fb,
                                        ((ki * g.KW + kj) * g.n_cchunks + cc) * CB, nt * BN);
                    }
                }
                __syncwarp();
                last_ph = (last_ph & ~(1u << s)) | (ph << s);
                used |= 1u << s;
                if (++cc == g.n_cchunks) {
                    cc = 0;
                    if (++kj == kw1) { kj = kw0; ++ki; }
                }
                if (++s == S) { s = 0; ph ^= 1; }
            }
        }
        // Every issued copy must have landed before the CTA exits (a stage that never
        // completes is reported; the others are still waited for).
        for (int st = 0; st < S; ++st)
            if ((used >> st) & 1u)
                if (!mbar_wait_warp(full0 + 8 * st, (last_ph >> st) & 1u, g.wait_limit) && lane == 0)
                    atomicExch(g.err, ERR_DRAIN);
        if (g.b_resident && !mbar_wait_warp(bfull, 0, g.wait_limit) && lane == 0) atomicExch(g.err, ERR_DRAIN);
    } else if (warp == 1) {
        // ---------------- MMA issuer (whole warp; one elected lane issues each MMA)
        const uint32_t idesc = make_idesc_i8(BN);
        // descriptors of stage 0 / B chunk 0; other stages, taps and chunks only move the
        // start address (16-byte units), so the issue loop is register adds.
        const uint64_t adesc0 = make_sdesc(smem_u32(sA), MODE == 2 ? 128 : CB);
        const uint64_t bdesc0 = make_sdesc(smem_u32(sB), CB);
        const uint64_t a_row_step = static_cast<uint64_t>((g.Wp * CB) >> 4);      // mode 1: next kernel row
        const uint64_t b_tap_step = static_cast<uint64_t>((g.n_cchunks * sb_stride) >> 4);
        const uint64_t a_stage_step = static_cast<uint64_t>(g.a_stage >> 4);
        const uint64_t b_chunk_step = static_cast<uint64_t>(sb_stride >> 4);
        const uint64_t xadesc0 = AUX ? make_sdesc(smem_u32(sA + g.aux_off), g.aux_kb) : 0;
        const uint64_t xbdesc = AUX ? make_sdesc(smem_u32(sBx), g.aux_kb) : 0;
        bool ok = !g.b_resident || mbar_wait_warp(bfull, 0, g.wait_limit);
        if (!ok && lane == 0) atomicExch(g.err, ERR_WAIT_FULL);
        int s = 0;
        uint32_t ph = 0;
        int buf = 0;
        uint32_t use_ph = 0;   // parity of the current use of accumulator `buf`
        for (int mt = blockIdx.x; ok && mt < g.m_tiles; mt += gridDim.x) {
            if (!mbar_wait_warp(acce0 + 8 * buf, use_ph ^ 1u, g.wait_limit)) {
                if (lane == 0) atomicExch(g.err, ERR_WAIT_EMPTY);
                break;
            }
            tc_fence_after();
            const uint32_t d = tmem + static_cast<uint32_t>(buf * g.acc_cols);
            int kh0 = 0, kh1 = 1, kw0 = 0, kw1 = 1;
            if (MODE == 0) tile_taps(g, mt, kh0, kh1, kw0, kw1);
            const int na = MODE == 0 ? (kh1 - kh0) * (kw1 - kw0) * g.n_cchunks : n_a;
            int ki = kh0, kj = kw0, cc = 0;   // mode 0: the K chunk's tap and channel chunk
            for (int ka = 0; ka < na; ++ka) {
                if (!mbar_wait_warp(full0 + 8 * s, ph, g.wait_limit)) {
                    if (lane == 0) atomicExch(g.err, ERR_WAIT_FULL);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint64_t da0 = adesc0 + static_cast<uint64_t>(s) * a_stage_step;
                if (MODE == 2) {
                    // A: 128-byte rows (two taps' 64 channels, 128-byte swizzle); B: the 64-byte chunks of
                    // taps 3i+j, resident.  Pair box: A bytes 0-63 x tap 3i, 64-127 x tap 3i+1; single-tap
                    // box: A bytes 0-63 x tap 3i+2.
                    const int t = 3 * (ka >> 1) + ((ka & 1) ? 2 : 0);
                    const uint64_t db = bdesc0 + static_cast<uint64_t>(t) * b_chunk_step;
                    mma_chunk_elect<2>(d, da0, db, idesc, ka != 0 ? 1u : 0u);
                    if ((ka & 1) == 0) mma_chunk_elect<2>(d, da0 + 4, db + b_chunk_step, idesc, 1u);
                } else if (MODE == 1 && g.KH == 1) {
                    // one tap (the stem GEMM over its bordered im2col rows): the block is the tile
                    mma_chunk_elect<CB / 32>(d, da0, bdesc0 + static_cast<uint64_t>(ka) * b_chunk_step, idesc,
                                             ka != 0 ? 1u : 0u);
                } else if (MODE == 1) {
                    // 3x3 taps (mode 1 is planned only for 3x3 convs and the 1x1 stem GEMM): the chunk's
                    // 9 x CB/32 MMAs from one asm block
                    mma_3x3_chunk<CB / 32>(d, da0, bdesc0 + static_cast<uint64_t>(ka) * b_chunk_step,
                                           static_cast<uint32_t>(a_row_step), static_cast<uint32_t>(b_tap_step), idesc,
                                           ka != 0 ? 1u : 0u);
                } else {
                    const int bc = (ki * g.KW + kj) * g.n_cchunks + cc;   // the chunk's index in the slab
                    const uint64_t db = bdesc0 + static_cast<uint64_t>(g.b_resident ? bc : s) * b_chunk_step;
                    mma_chunk_elect<CB / 32>(d, da0, db, idesc, ka != 0 ? 1u : 0u);
                    if (++cc == g.n_cchunks) {
                        cc = 0;
                        if (++kj == kw1) { kj = kw0; ++ki; }
                    }
                }
                if (AUX && ka == 0) {
                    const uint32_t dx = d + static_cast<uint32_t>(g.aux_col);
                    const uint64_t xa = xadesc0 + static_cast<uint64_t>(s) * a_stage_step;
                    if (g.aux_kb == 32) mma_chunk_elect<1>(dx, xa, xbdesc, idesc, 0u);
                    else if (g.aux_kb == 64) mma_chunk_elect<2>(dx, xa, xbdesc, idesc, 0u);
                    else mma_chunk_elect<4>(dx, xa, xbdesc, idesc, 0u);
                }
                mma_commit_elect(empty0 + 8 * s);
                if (++s == S) { s = 0; ph ^= 1; }
            }
            if (!ok) break;
            mma_commit_elect(accf0 + 8 * buf);
            if (++buf == NA) { buf = 0; use_ph ^= 1u; }
        }
        // all MMAs of this warp complete before TMEM can be released
        mma_commit_elect(donebar);
        if (!mbar_wait_warp(donebar, 0, g.wait_limit) && lane == 0) atomicExch(g.err, ERR_WAIT_ACC);
    } else {
        // ---------------- epilogue: TMEM lanes 32*(warp%4) .. +31 = tile rows.
        // Warps form NG groups; group gi takes tiles t = gi (mod NG), held in accumulator
        // t % NA, so NA tiles are in flight.  Inside a group the warps of a quadrant take
        // interleaved 16-column groups.
        if (g.b_packed) {
            // Packed W4 slab -> int8 codes in the swizzled layout TMA would have written:
            // chunk kc holds rows n < BN of CB bytes, and the 16-byte granule of byte offset
            // o = n*CB + 16j sits at o ^ (((o >> 7) & m) << 4) (m = 7 / 3 / 1 for the 128 /
            // 64 / 32-byte swizzle; chunks are 1024-byte aligned).  Rows past the weight
            // matrix are zero, as TMA's out-of-bounds fill.  The weights are constants:
            // this runs before griddepcontrol.wait, under the previous kernel's tail.
            constexpr uint32_t kSwz = CB == 128 ? 7u : (CB == 64 ? 3u : 1u);
            constexpr int kGran = CB / 16;
            const int per_chunk = BN * kGran;
            const int total = g.n_kchunks * per_chunk;
            for (int u = static_cast<int>(threadIdx.x) - 64; u < total; u += 32 * kEpiWarps) {
                const int kc = u / per_chunk;
                const int rem = u - kc * per_chunk;
                const int n = rem / kGran, j = rem - (rem / kGran) * kGran;
                const int row = nt * BN + n;
                uint4 v = make_uint4(0u, 0u, 0u, 0u);
                if (row < g.w_rows) {
                    const uint2 p = __ldg(reinterpret_cast<const uint2*>(
                        g.w4 + static_cast<size_t>(row) * g.w4_ld + kc * (CB / 2) + 8 * j));
                    unpack_w4(p.x, v.x, v.y);
                    unpack_w4(p.y, v.z, v.w);
                }
                const uint32_t o = static_cast<uint32_t>(n * CB + 16 * j);
                *reinterpret_cast<uint4*>(sB + kc * sb_stride + (o ^ (((o >> 7) & kSwz) << 4))) = v;
            }
            fence_proxy_async_smem();
            named_bar_sync(1, 32 * kEpiWarps);
            if (threadIdx.x == 64) mbar_arrive(bfull);
        }
        if constexpr (FBN > 0) {
            epilogue_fast<CB, NOUT, RES, F32, AUX, FBN>(g, e, cc, tmem, accf0, acce0, warp, lane);
        } else {
        const int ew = warp - 2;
        const int gi = ew / group_warps;
        const int quad = warp & 3;
        const int slice = (ew % group_warps) >> 2;
        const int kSlices = group_warps / 4;
        const int r = quad * 32 + lane;
        const int tw = g.TW, th = g.TH;
        const int rn = r / (tw * th), rh = (r / tw) % th, rw = r % tw;
        const bool in_tile = r < tw * th * g.TN;
        const int tile_end = min(e.cout, (nt + 1) * BN);
        const int ncg = bn32 / 32;   // 32-column groups, each handled as two 16-column halves
        constexpr int n_out = NOUT;
        // One quantizer form (clamp to [y_lo, y_hi]) for every output.  Codes only (no fp32
        // values kept): the conv's activation (no residual) or the post-add ReLU (residual)
        // is folded into that clamp.  With fp32 values kept, the values are final and the
        // lower bound is 0 where they cannot be negative (the clamp then changes nothing).
        constexpr bool kFold = !RES && !F32 && !AUX;      // activation folded
        constexpr bool kFoldPost = RES && !F32;           // post-add ReLU folded
        const bool nonneg = RES ? e.post == 1 : e.act != 0;
        QParams qx0 = e.q0, qx1 = e.q1;
        if (kFold) {
            qx0 = fold_act(e.q0, e.act);
            qx1 = fold_act(e.q1, e.act);
        } else if (nonneg) {
            qx0.y_lo = 0.0f;
            qx1.y_lo = 0.0f;
        }
        // the value a code encodes, for the per-value path of partial channel groups
        auto final_val = [&](float v) {
            if (kFold) return apply_act(v, e.act);
            if (kFoldPost && e.post == 1) return fmaxf(v, 0.0f);
            return v;
        };
        griddep_wait();   // residuals are earlier kernels' outputs
        // output position of this thread's row r in M tile mt: image n, row h, column w,
        // bordered code row pq, fp32 row pf
        // (bordered positions and tile indices stay below 2^32: the host limits the batch)
        auto position = [&](int mt, int& n, int& h, int& w, bool& valid, size_t& pq, size_t& pf) {
            if (MODE == 1) {
                const uint32_t q = static_cast<uint32_t>(mt) * 128u + static_cast<uint32_t>(r);
                const uint32_t nn = fdiv(q, g.fd_img);
                const uint32_t rem = q - nn * g.fd_img.d;
                const uint32_t hb = fdiv(rem, g.fd_wp);
                n = static_cast<int>(nn);
                h = static_cast<int>(hb) - 1;
                w = static_cast<int>(rem - hb * g.fd_wp.d) - 1;
                valid = n < g.N && h >= 0 && h < g.OH && w >= 0 && w < g.OW;
                pq = q;
            } else {
                const uint32_t rest = fdiv(static_cast<uint32_t>(mt), g.fd_tiles_w);
                const uint32_t tw_i = static_cast<uint32_t>(mt) - rest * g.fd_tiles_w.d;
                const uint32_t nb = fdiv(rest, g.fd_tiles_h);
                n = static_cast<int>(nb) * g.TN + rn;
                h = static_cast<int>(rest - nb * g.fd_tiles_h.d) * g.TH + rh;
                w = static_cast<int>(tw_i) * g.TW + rw;
                valid = in_tile && n < g.N && h < g.OH && w < g.OW;
                pq = (static_cast<size_t>(n) * (g.OH + 2) + h + 1) * (g.OW + 2) + w + 1;
            }
            pf = (static_cast<size_t>(n) * g.OH + h) * g.OW + w;
        };
        if (NG == 1) {
            // Column-stationary epilogue (N tile of 49..64 channels, one group): warp
            // (quad, k) owns channels [16k, 16k+16) of its 32 rows in every tile, so its
            // dequantization constants stay in registers for the whole kernel.
            const int k = ew >> 2;
            const int ch = nt * BN + k * 16;
            const bool active = ch < tile_end;   // warp-uniform
            const int nv = min(16, tile_end - ch);
            float2 fbr[16], afbr[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                fbr[j] = cc.fb[ch + j];
                if (AUX) afbr[j] = cc.aux_fb[ch + j];
            }
            int buf = 0;
            uint32_t use = 0;   // parity of the current use of accumulator `buf`
            for (int mt = blockIdx.x; mt < g.m_tiles; mt += gridDim.x) {
                int n, h, w;
                bool valid;
                size_t pq, pf;
                position(mt, n, h, w, valid, pq, pf);
                float res[16];
                if (RES && !AUX && valid && active) load_res16(e, pf, ch, nv, res);
                if (!mbar_wait(accf0 + 8 * buf, use & 1u, g.wait_limit)) {
                    atomicExch(g.err, ERR_WAIT_ACC);
                    break;
                }
                tc_fence_after();
                if (active) {
                    const uint32_t trow =
                        tmem + static_cast<uint32_t>(buf * g.acc_cols) + (static_cast<uint32_t>(quad * 32) << 16);
                    uint32_t v[16], vx[16];
                    tmem_ld16(trow + k * 16, v);
                    if (AUX) tmem_ld16(trow + static_cast<uint32_t>(g.aux_col) + k * 16, vx);
                    tmem_wait_ld();
                    if (valid) {
                        float y[16];
                        dequant16(v, fbr, e.act, y, !e.acc_small);
                        if (AUX) dequant16(vx, afbr, e.aux_act, res, false);   // aux K <= 128
                        finish16<RES, F32, !kFoldPost>(e, pf, ch, nv, y, res);
#pragma unroll
                        for (int o = 0; o < 2; ++o) {
                            if (o >= n_out) continue;
                            if (!code_kept(e, o, h, w)) continue;
                            int8_t* qp = code_ptr(e, o, pq, n, ch, h, w);
                            if (nv == 16) {
                                uint32_t w4[4];
                                quant16q<true>(y, o == 0 ? qx0 : qx1, o == 0 ? e.s0 : e.s1, w4);
                                st_v4(qp, make_uint4(w4[0], w4[1], w4[2], w4[3]));
                            } else {
                                const float inv = o == 0 ? e.inv0 : e.inv1;
                                const double s = o == 0 ? e.s0 : e.s1;
#pragma unroll
                                for (int j = 0; j < 16; ++j)
                                    if (j < nv) qp[j] = sat8(quant_code(final_val(y[j]), inv, s));
                            }
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_relaxed(acce0 + 8 * buf);
                if (++buf == NA) {
                    buf = 0;
                    use ^= 1u;
                }
            }
        } else {
        // tiles t = gi, gi + NG, ...: accumulator t % NA (NG divides NA), parity (t / NA) & 1
        int buf = gi;
        uint32_t use = 0;
        for (int mt = blockIdx.x + gi * gridDim.x; mt < g.m_tiles; mt += NG * gridDim.x) {
            int n, h, w;
            bool valid;
            size_t pq, pf;
            position(mt, n, h, w, valid, pq, pf);
            // the residual does not depend on the MMAs: fetch the first half before waiting
            float res[16];
            {
                const int c0 = nt * BN + slice * 32;
                if (RES && !AUX && valid && slice < ncg && c0 < tile_end)
                    load_res16(e, pf, c0, min(16, tile_end - c0), res);
            }
            if (!mbar_wait(accf0 + 8 * buf, use & 1u, g.wait_limit)) {
                atomicExch(g.err, ERR_WAIT_ACC);
                break;
            }
            tc_fence_after();
            const uint32_t trow = tmem + static_cast<uint32_t>(buf * g.acc_cols) + (static_cast<uint32_t>(quad * 32) << 16);
            for (int cg = slice; cg < ncg; cg += kSlices) {
                const int c0 = nt * BN + cg * 32;
                const int nv32 = min(32, tile_end - c0);   // valid channels of this 32-group (may be <= 0)
                uint32_t wq[2][8];                          // codes of both halves, per output
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    uint32_t v[16], vx[16];
                    __syncwarp();   // tcgen05.ld is .sync.aligned: reconverge after the per-lane stores
                    tmem_ld16(trow + cg * 32 + hh * 16, v);
                    if (AUX) tmem_ld16(trow + static_cast<uint32_t>(g.aux_col) + cg * 32 + hh * 16, vx);
                    tmem_wait_ld();
                    const int ch = c0 + hh * 16;
                    const int nv = min(16, tile_end - ch);
                    if (!valid || nv <= 0) continue;
                    float y[16];
                    dequant16(v, cc.fb + ch, kFold ? 0 : e.act, y, !e.acc_small);
                    if (AUX) dequant16(vx, cc.aux_fb + ch, e.aux_act, res, false);   // aux K <= 128
                    finish16<RES, F32, !kFoldPost>(e, pf, ch, nv, y, res);
                    // prefetch the next residual half of this warp
                    {
                        const int cn = hh == 0 ? ch + 16 : c0 + 32 * kSlices;
                        if (RES && !AUX && (hh == 0 || cg + kSlices < ncg) && cn < tile_end)
                            load_res16(e, pf, cn, min(16, tile_end - cn), res);
                    }
#pragma unroll
                    for (int o = 0; o < 2; ++o) {
                        if (o >= n_out) continue;
                        const float inv = o == 0 ? e.inv0 : e.inv1;
                        const double s = o == 0 ? e.s0 : e.s1;
                        if (nv32 == 32) {
                            uint32_t w4[4];
                            quant16q<true>(y, o == 0 ? qx0 : qx1, s, w4);
#pragma unroll
                            for (int j = 0; j < 4; ++j) wq[o][hh * 4 + j] = w4[j];
                        } else {
                            if (!code_kept(e, o, h, w)) continue;
                            int8_t* qp = code_ptr(e, o, pq, n, ch, h, w);
                            if (NOUT <= 1 && !e.dcr_oc) {
                                // Partial group: channels past tile_end are the code row's padding
                                // (only the last N tile is partial, and ldq is cout rounded up to
                                // 32); their constants are zero, so they dequantize to 0 and get
                                // code 0, the padding's value: all 16 codes go out in one store.
                                // (Single-output kernels only: in two-output ones the extra path
                                // costs register spills.)
                                uint32_t w4[4];
                                quant16q<true>(y, o == 0 ? qx0 : qx1, s, w4);
                                st_v4(qp, make_uint4(w4[0], w4[1], w4[2], w4[3]));
                            } else {
                                // positionally decomposed: channels past a position belong to another
#pragma unroll
                                for (int j = 0; j < 16; ++j)
                                    if (j < nv) qp[j] = sat8(quant_code(final_val(y[j]), inv, s));
                            }
                        }
                    }
                }
                // full 32-channel groups: one 32-byte (full-sector) store per output
                if (valid && nv32 == 32) {
#pragma unroll
                    for (int o = 0; o < 2; ++o)
                        if (o < n_out && code_kept(e, o, h, w))
                            st_v8(reinterpret_cast<uint32_t*>(code_ptr(e, o, pq, n, c0, h, w)), wq[o]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_relaxed(acce0 + 8 * buf);
            if ((buf += NG) >= NA) {
                buf -= NA;
                use ^= 1u;
            }
        }
        }
        }   // general epilogue
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, NA * g.acc_cols);
}

// ------------------------------------------------------------------ stem im2col

// Normalisation of 8-bit pixels (CIFAR-10 records) into the network's fp32 input, in
// the float32 operations of one of the reference's two input paths (per channel c,
// px the pixel as a float, m[c] = mean*255 and d[c] as below, all float32):
//   kNormDiv: x = (px - m) / d, d = std*255        (06-gpu-int8/cpp/ref_e2e.py:261-276)
//   kNormMul: x = ((px / 255) * 255 - m) * d,
//             d = 1 / (std*255)                      (06-gpu-int8/cpp/main.cpp:245-261)
// each operation rounded to nearest (no contraction), as numpy and the reference's
// host loop compute them.
enum { kNormDiv = 0, kNormMul = 1 };
struct U8Norm {
    int mode;
    float m[4], d[4];
};
__device__ __forceinline__ float normalize_px(uint32_t px, int c, const U8Norm& nm) {
    const float v = static_cast<float>(px);
    if (nm.mode == kNormMul) return __fmul_rn(__fsub_rn(__fmul_rn(__fdiv_rn(v, 255.0f), 255.0f), nm.m[c]), nm.d[c]);
    return __fdiv_rn(__fsub_rn(v, nm.m[c]), nm.d[c]);
}

// x: fp32 NCHW [N][C][H][W] (U8: 8-bit pixels [N][C][H][W], normalised as above);
// out: int8 rows of a bordered [N][OH+2][OW+2][kpad]
// map (border rows are never written and stay zero) with k = (i*KW + j)*C + c,
// codes of the stem's scale, zero for out-of-image taps and k >= KH*KW*C.
// One CTA per band of `rows` output rows of one image.  The input band is read
// once (consecutive threads take consecutive band elements, 16 loads in flight
// per thread) and quantized once into shared memory with its zero padding; a
// table maps k to its offset in the band; then
// each thread assembles the kpad-byte im2col row of one output pixel and writes
// it with 16-byte stores (consecutive pixels: consecutive rows).
// U8: a pixel's code depends only on (channel, value), so the CTA first fills a
// [C][256] code table (normalise + exact quantize of every value) and the band is
// then a byte gather from it: the decode, normalisation and quantization of the
// network input happen here, and the host sends 1 byte per input value instead of 4.
template <bool U8>
__global__ void stem_im2col_kernel(const void* __restrict__ xin, int8_t* __restrict__ out, int N, int C, int H,
                                   int W, int OH, int OW, int KH, int KW, int SH, int SW, int PH, int PW,
                                   int kpad, int rows, float inv, double s, U8Norm nm) {
    griddep_launch();
    // [C][band_h][band_w], then int koff[kpad], then (U8) int8 lut[C][256]
    extern __shared__ __align__(16) int8_t band[];
    const int bands = (OH + rows - 1) / rows;
    const int n = blockIdx.x / bands;
    const int r0 = (blockIdx.x - n * bands) * rows;
    const int r1 = min(OH, r0 + rows);
    const int band_h = (rows - 1) * SH + KH;
    const int band_w = (OW - 1) * SW + KW;
    const int band_bytes = C * band_h * band_w;
    int* koff = reinterpret_cast<int*>(band + ((band_bytes + 15) & ~15));
    int8_t* lut = reinterpret_cast<int8_t*>(koff + kpad);
    if (U8) {   // depends on nothing an earlier kernel writes: built before the dependency wait
        for (int i = threadIdx.x; i < C * 256; i += blockDim.x)
            lut[i] = static_cast<int8_t>(sat8(quant_code(normalize_px(i & 255, i >> 8, nm), inv, s)));
    }
    griddep_wait();
    const int K = KH * KW * C;
    for (int k = threadIdx.x; k < kpad; k += blockDim.x) {
        int o = -1;
        if (k < K) {
            const int c = k % C, tap = k / C;
            o = (c * band_h + tap / KW) * band_w + tap % KW;
        }
        koff[k] = o;
    }
    // The band, element e = (c * band_h + bh) * band_w + bw, in rounds of 16 elements
    // per thread: all 16 loads are issued before the first is quantized, so a round
    // waits for one memory latency (a warp per band row, row after row, waited for one
    // per row).  Out-of-image elements are the zero padding.
    const int ih0 = r0 * SH - PH, iw0 = -PW;
    constexpr int kRound = 16;
    if (!U8) {
        const float* xn = static_cast<const float*>(xin) + static_cast<size_t>(n) * C * H * W;
        for (int e0 = 0; e0 < band_bytes; e0 += kRound * static_cast<int>(blockDim.x)) {
            float v[kRound];
#pragma unroll
            for (int m = 0; m < kRound; ++m) {
                const int e = e0 + m * static_cast<int>(blockDim.x) + static_cast<int>(threadIdx.x);
                const int rr = e / band_w, bw = e - rr * band_w;
                const int c = rr / band_h, bh = rr - c * band_h;
                const int ih = ih0 + bh, iw = iw0 + bw;
                const bool in = e < band_bytes && ih >= 0 && ih < H && iw >= 0 && iw < W;
                v[m] = in ? __ldg(xn + (static_cast<size_t>(c) * H + ih) * W + iw) : 0.0f;
            }
#pragma unroll
            for (int m = 0; m < kRound; ++m) {
                const int e = e0 + m * static_cast<int>(blockDim.x) + static_cast<int>(threadIdx.x);
                if (e < band_bytes) band[e] = static_cast<int8_t>(sat8(quant_code(v[m], inv, s)));
            }
        }
    } else {
        const uint8_t* xn = static_cast<const uint8_t*>(xin) + static_cast<size_t>(n) * C * H * W;
        __syncthreads();   // the code table
        for (int e0 = 0; e0 < band_bytes; e0 += kRound * static_cast<int>(blockDim.x)) {
            int v[kRound];   // lut index, or -1 for the zero padding
#pragma unroll
            for (int m = 0; m < kRound; ++m) {
                const int e = e0 + m * static_cast<int>(blockDim.x) + static_cast<int>(threadIdx.x);
                const int rr = e / band_w, bw = e - rr * band_w;
                const int c = rr / band_h, bh = rr - c * band_h;
                const int ih = ih0 + bh, iw = iw0 + bw;
                const bool in = e < band_bytes && ih >= 0 && ih < H && iw >= 0 && iw < W;
                v[m] = in ? (c << 8) + __ldg(xn + (static_cast<size_t>(c) * H + ih) * W + iw) : -1;
            }
#pragma unroll
            for (int m = 0; m < kRound; ++m) {
                const int e = e0 + m * static_cast<int>(blockDim.x) + static_cast<int>(threadIdx.x);
                if (e < band_bytes) band[e] = v[m] >= 0 ? lut[v[m]] : static_cast<int8_t>(0);
            }
        }
    }
    __syncthreads();
    const int npix = (r1 - r0) * OW;
    int8_t* obase = out + ((static_cast<size_t>(n) * (OH + 2) + r0 + 1) * (OW + 2) + 1) * kpad;
    // 16 bytes of every pixel's row at a time: their 16 band offsets stay in registers
    // for all of this thread's pixels
    for (int k0 = 0; k0 < kpad; k0 += 16) {
        int ko[16];
#pragma unroll
        for (int b = 0; b < 16; ++b) ko[b] = koff[k0 + b];
        for (int p = threadIdx.x; p < npix; p += blockDim.x) {
            const int ohl = p / OW, ow = p - (p / OW) * OW;
            const int8_t* bp = band + ohl * SH * band_w + ow * SW;
            uint32_t wv[4];
#pragma unroll
            for (int wd = 0; wd < 4; ++wd) {
                uint32_t packed = 0;
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const int o = ko[wd * 4 + b];
                    const uint32_t q = o >= 0 ? static_cast<uint8_t>(bp[o]) : 0u;
                    packed |= q << (8 * b);
                }
                wv[wd] = packed;
            }
            st_v4(obase + static_cast<size_t>(ohl * (OW + 2) + ow) * kpad + k0, make_uint4(wv[0], wv[1], wv[2], wv[3]));
        }
    }
}

// The CIFAR stem (3 channels, 3x3, stride 1, pad 1, 32-byte im2col rows), same output as
// stem_im2col_kernel: the band is kept pixel-major, [band_h][band_w][3] codes, so the 27
// codes of output pixel (h, w) -- k = (i*3 + j)*3 + c -- are three runs of 9 consecutive
// bytes, one per kernel row i, starting at ((h + i)*band_w + w)*3.  Each run is read as three
// aligned words and funnel-shifted into place (no per-byte loads), and the row goes out as two
// 16-byte stores.  Band element indices are split by multiply-high division (fd_bw = band_w,
// fd_bh = band_h).  U8: 8-bit pixels through the per-CTA code table, as in stem_im2col_kernel.
template <bool U8>
__global__ void stem_im2col3_kernel(const void* __restrict__ xin, int8_t* __restrict__ out, int N, int H, int W,
                                    int rows, FastDiv fd_bw, FastDiv fd_bh, float inv, double s, U8Norm nm) {
    griddep_launch();
    // [band_h][band_w][3] codes, 16 spare bytes (the last run's word reads), then (U8) int8 lut[3][256]
    extern __shared__ __align__(16) int8_t band[];
    const int bands = (H + rows - 1) / rows;
    const int n = blockIdx.x / bands;
    const int r0 = (blockIdx.x - n * bands) * rows;
    const int r1 = min(H, r0 + rows);
    const int band_w = static_cast<int>(fd_bw.d), band_h = static_cast<int>(fd_bh.d);
    const int band_bytes = band_h * band_w * 3;
    int8_t* lut = band + ((band_bytes + 16 + 15) & ~15);
    if (U8) {   // depends on nothing an earlier kernel writes: built before the dependency wait
        for (int i = threadIdx.x; i < 3 * 256; i += blockDim.x)
            lut[i] = static_cast<int8_t>(sat8(quant_code(normalize_px(i & 255, i >> 8, nm), inv, s)));
    }
    if (threadIdx.x < 16) band[band_bytes + threadIdx.x] = 0;
    griddep_wait();
    if (U8) __syncthreads();   // the code table
    // band element e = (c * band_h + bh) * band_w + bw: consecutive threads read consecutive
    // input columns; 16 loads in flight per thread; out-of-image elements are code 0
    const int ih0 = r0 - 1;
    constexpr int kRound = 16;
    const size_t img = static_cast<size_t>(n) * 3 * H * W;
    for (int e0 = 0; e0 < band_bytes; e0 += kRound * static_cast<int>(blockDim.x)) {
        int dst[kRound];
        float v[kRound];
        int li[kRound];
#pragma unroll
        for (int m = 0; m < kRound; ++m) {
            const int e = e0 + m * static_cast<int>(blockDim.x) + static_cast<int>(threadIdx.x);
            const uint32_t rr = fdiv(static_cast<uint32_t>(e), fd_bw);
            const int bw = e - static_cast<int>(rr) * band_w;
            const uint32_t c = fdiv(rr, fd_bh);
            const int bh = static_cast<int>(rr) - static_cast<int>(c) * band_h;
            const int ih = ih0 + bh, iw = bw - 1;
            const bool in = e < band_bytes && ih >= 0 && ih < H && iw >= 0 && iw < W;
            const size_t gi = img + (static_cast<size_t>(c) * H + ih) * W + iw;
            dst[m] = e < band_bytes ? (bh * band_w + bw) * 3 + static_cast<int>(c) : -1;
            if (U8) {
                li[m] = in ? static_cast<int>(c << 8) + __ldg(static_cast<const uint8_t*>(xin) + gi) : -1;
            } else {
                v[m] = in ? __ldg(static_cast<const float*>(xin) + gi) : 0.0f;
            }
        }
#pragma unroll
        for (int m = 0; m < kRound; ++m) {
            if (dst[m] < 0) continue;
            if (U8) band[dst[m]] = li[m] >= 0 ? lut[li[m]] : static_cast<int8_t>(0);
            else band[dst[m]] = static_cast<int8_t>(sat8(quant_code(v[m], inv, s)));
        }
    }
    __syncthreads();
    const int npix = (r1 - r0) * W;
    int8_t* obase = out + ((static_cast<size_t>(n) * (H + 2) + r0 + 1) * (W + 2) + 1) * 32;
    const uint32_t* bw32 = reinterpret_cast<const uint32_t*>(band);
    for (int p = threadIdx.x; p < npix; p += blockDim.x) {
        const int hl = p / W, w = p - (p / W) * W;
        uint32_t s0[3], s1[3], b8[3];
#pragma unroll
        for (int i = 0; i < 3; ++i) {
            const int off = ((hl + i) * band_w + w) * 3;
            const int a = off >> 2;
            const uint32_t sh = static_cast<uint32_t>(off & 3) * 8u;
            const uint32_t w0 = bw32[a], w1 = bw32[a + 1], w2 = bw32[a + 2];
            s0[i] = __funnelshift_r(w0, w1, sh);   // bytes 0..3 of the run
            s1[i] = __funnelshift_r(w1, w2, sh);   // bytes 4..7
            b8[i] = (w2 >> sh) & 0xFFu;            // byte 8
        }
        // row bytes: run 0 at 0..8, run 1 at 9..17, run 2 at 18..26, zeros at 27..31
        uint4 lo, hi;
        lo.x = s0[0];
        lo.y = s1[0];
        lo.z = b8[0] | (s0[1] << 8);
        lo.w = (s0[1] >> 24) | (s1[1] << 8);
        hi.x = (s1[1] >> 24) | (b8[1] << 8) | (s0[2] << 16);
        hi.y = (s0[2] >> 16) | (s1[2] << 16);
        hi.z = (s1[2] >> 16) | (b8[2] << 16);
        hi.w = 0u;
        int8_t* o = obase + static_cast<size_t>(hl * (W + 2) + w) * 32;
        st_v4(o, lo);
        st_v4(o + 16, hi);
    }
}

// ------------------------------------------------------------------ depthwise conv

// Depthwise kxk conv over bordered int8 codes [N][H+2][W+2][ldi] (C channels),
// int32 accumulation, then the shared exact epilogue.  One thread per
// (position, 4 channels); weights w[tap][C] int8.
__global__ void dw_conv_kernel(const int8_t* __restrict__ in, int ldi, const int8_t* __restrict__ w, int N, int H,
                               int W, int C, int OH, int OW, int KH, int KW, int SH, int SW, int PH, int PW,
                               const EpiParams e) {
    griddep_launch();
    griddep_wait();
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
                const char4 xv = *reinterpret_cast<const char4*>(
                    in + ((static_cast<size_t>(n) * (H + 2) + ih + 1) * (W + 2) + iw + 1) * ldi + c0);
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
                y[b] = __fadd_rn(y[b], e.residual[f32_off(p, c0 + b, C)]);
                if (e.post == 1) y[b] = fmaxf(y[b], 0.0f);
            }
        }
        if (e.out_f32)
            for (int b = 0; b < nv; ++b) e.out_f32[f32_off(p, c0 + b, C)] = y[b];
        const size_t pq = (static_cast<size_t>(n) * (OH + 2) + oh + 1) * (OW + 2) + ow + 1;
        if (e.out_q0)
            for (int b = 0; b < nv; ++b) e.out_q0[pq * e.ldq0 + c0 + b] = sat8(quant_code(y[b], e.inv0, e.s0));
        if (e.out_q1)
            for (int b = 0; b < nv; ++b) e.out_q1[pq * e.ldq1 + c0 + b] = sat8(quant_code(y[b], e.inv1, e.s1));
    }
}

// Depthwise 3x3 conv, padding 1, stride S (1 or 2), over bordered int8 codes
// [N][H+2][W+2][ldi]: the reference's depthwise conv (ref_int8.py conv with
// groups == cin) for the 3x3 shapes MobileNetV2 uses.
//
// Staging: the input goes to shared memory by bulk copies (cp.async.bulk) in
// n_stages stages, issued by one producer warp (the block's last) behind
// full/empty mbarriers, so the copies run ahead of the arithmetic and consumer
// warps never wait on one another.  A unit is either a band of R output rows of
// one image (the S*(R-1)+3 bordered input rows it reads, contiguous in the
// bordered layout) or k whole images (R = OH; all H+2 bordered rows of each).
// Persistent CTAs take units blockIdx.x, +gridDim.x, ...
//
// Arithmetic: item = (strip of T horizontally adjacent output positions, word
// g of 4 channels), item index strip * G4 + g: consecutive lanes read
// consecutive 4-byte words of the same pixels.  The consumer count is a
// multiple of G4, so a thread's g never changes and its weights (12 words) and
// dequantization constants (4 pairs) stay in registers.  Weight word (j, c) of
// the host table is column j of channel 4g+c's 3x3 kernel: bytes (w[0][j],
// w[1][j], w[2][j], 0).  Each of the S*(T-1)+3 input columns of a strip is
// loaded once (3 words: rows 0-2) and transposed with byte permutes into one
// word per channel holding the column's 3 taps, which every position of the
// strip that uses the column multiplies by the matching weight column with one
// dp4a.  Integer sums are exact, so the order of taps does not change the
// accumulator; |acc| <= 9 * 128 * 128 < 2^22, so the accumulators start at the
// float-conversion bias 0x4B400000 and their final bits are already those of
// 1.5*2^23 + acc (no range check, no add in the epilogue).
//
// Epilogue: y = fadd(fmul(float(acc), factor), bias), then the activation and
// the quantizer's clamp as one clamp: relu6 then clip to [y_lo, y_hi] is
// clip(y, 0, min(6, y_hi)) (y_lo < 0), so codes are unchanged.  Channels c >= C
// have zero weights and constants: their codes are 0, written into the code
// row's padding (ldq >= 4 G4).  Convs with a residual, an fp32 output or a
// subsampled code output use dw_conv_kernel.
struct DwGeom {
    int G4, C, H, W, OH, OW, ldi, N;
    int R;            // output rows per unit
    int k_img;        // images per unit (> 1 only when R == OH)
    int rows_img;     // bordered input rows staged per image
    int bands;        // OH / R
    int n_units;
    int stage_bytes;  // bytes per stage (multiple of 128)
    int n_stages;
    int strips;       // strips per output row (OW / T)
    FastDiv fd_strips, fd_rs, fd_bands;   // strips, R * strips, bands
    int* err;              // the engine's device error word
    long long wait_limit;  // bounded-wait limit, clock cycles
    int w_packed;          // W4 conv: the weight table holds 16-bit words of 3 int4 codes (see dw3x3_kernel)
};

constexpr int kDwMaxStages = 4;
constexpr int kDwMaxConsumers = 640;   // consumer threads per CTA (+ one producer warp)
constexpr int kDwBulkChunk = 16384;    // bytes per bulk copy instruction

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
                 : "memory");
}

// First image and first output row of unit u, and the byte range it stages.
__device__ __forceinline__ void dw_unit(const DwGeom& d, int S, uint32_t u, int& n0, int& r0, int& k,
                                        size_t& src_off, uint32_t& bytes) {
    const size_t row = static_cast<size_t>(d.W + 2) * d.ldi;
    if (d.k_img == 1) {
        n0 = static_cast<int>(fdiv(u, d.fd_bands));
        r0 = (static_cast<int>(u) - n0 * d.bands) * d.R;
        k = 1;
        src_off = (static_cast<size_t>(n0) * (d.H + 2) + static_cast<size_t>(r0) * S) * row;
        bytes = static_cast<uint32_t>(d.rows_img * row);
    } else {
        n0 = static_cast<int>(u) * d.k_img;
        r0 = 0;
        k = min(d.k_img, d.N - n0);
        src_off = static_cast<size_t>(n0) * (d.H + 2) * row;
        bytes = static_cast<uint32_t>(k * (d.H + 2) * row);
    }
}

// Column word x_i (row i, 4 channels) -> y[c] = (x0.b_c, x1.b_c, x2.b_c, *).
// The fourth byte meets a zero weight byte.
__device__ __forceinline__ void col_transpose3(uint32_t x0, uint32_t x1, uint32_t x2, uint32_t (&y)[4]) {
    const uint32_t a = __byte_perm(x0, x1, 0x5140);   // x0.b0 x1.b0 x0.b1 x1.b1
    const uint32_t b = __byte_perm(x0, x1, 0x7362);   // x0.b2 x1.b2 x0.b3 x1.b3
    y[0] = __byte_perm(a, x2, 0x5410);                // a.b0 a.b1 x2.b0 (x2.b1)
    y[1] = __byte_perm(a, x2, 0x6532);                // a.b2 a.b3 x2.b1 (x2.b2)
    y[2] = __byte_perm(b, x2, 0x7610);                // b.b0 b.b1 x2.b2 (x2.b3)
    y[3] = __byte_perm(b, x2, 0x7732);                // b.b2 b.b3 x2.b3 (x2.b3)
}

template <int T, int S, int ACT>
__global__ void __launch_bounds__(kDwMaxConsumers + 32, 1) dw3x3_kernel(const int8_t* __restrict__ in,
                                                                        const uint4* __restrict__ wt, const DwGeom d,
                                                                        const EpiParams e) {
    extern __shared__ __align__(128) uint8_t dw_smem[];
    __shared__ __align__(8) uint64_t bars[2 * kDwMaxStages];   // full[s], empty[s]
    griddep_launch();
    const int n_cons = static_cast<int>(blockDim.x) - 32;
    const uint32_t bar0 = smem_u32(&bars[0]);
    if (threadIdx.x == 0) {
        for (int s = 0; s < d.n_stages; ++s) {
            mbar_init(bar0 + 8 * s, 1);
            mbar_init(bar0 + 8 * (kDwMaxStages + s), n_cons / 32);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (static_cast<int>(threadIdx.x) >= n_cons) {
        // ---- producer warp
        griddep_wait();
        if (threadIdx.x != static_cast<unsigned>(n_cons)) return;
        int issued = 0;
        for (uint32_t u = blockIdx.x; u < static_cast<uint32_t>(d.n_units); u += gridDim.x, ++issued) {
            const int stage = issued % d.n_stages;
            if (issued >= d.n_stages &&
                !mbar_wait(bar0 + 8 * (kDwMaxStages + stage), static_cast<uint32_t>(issued / d.n_stages - 1) & 1u,
                           d.wait_limit)) {
                atomicExch(d.err, ERR_WAIT_EMPTY);
                break;
            }
            int n0, r0, k;
            size_t off;
            uint32_t bytes;
            dw_unit(d, S, u, n0, r0, k, off, bytes);
            const uint32_t bar = bar0 + 8 * stage;
            const uint32_t dst = smem_u32(dw_smem + stage * d.stage_bytes);
            mbar_expect_tx(bar, bytes);
            for (uint32_t b = 0; b < bytes; b += kDwBulkChunk)
                bulk_load(dst + b, in + off + b, min(bytes - b, static_cast<uint32_t>(kDwBulkChunk)), bar);
        }
        // let the copies issued last land before the CTA's shared memory goes away
        // (already complete unless a consumer gave up early)
        for (int j = max(0, issued - d.n_stages); j < issued; ++j)
            if (!mbar_wait(bar0 + 8 * (j % d.n_stages), static_cast<uint32_t>(j / d.n_stages) & 1u, d.wait_limit))
                atomicExch(d.err, ERR_DRAIN);
        return;
    }

    // ---- consumers
    const int G4 = d.G4;
    const uint32_t g = threadIdx.x % static_cast<uint32_t>(G4);
    const int c0 = 4 * static_cast<int>(g);
    uint32_t w[12];   // w[3 j + ... ]: column j, channel c at w[4 j + c]
    if (d.w_packed) {
        // W4: 12 16-bit words per group (24 bytes), word 4j + c = codes (w0j, w1j, w2j) of
        // channel 4g + c as nibbles 0-2; spread to bytes and sign-extended
        const uint2* p = reinterpret_cast<const uint2*>(wt) + 3 * g;
        const uint2 a = __ldg(p), b = __ldg(p + 1), c = __ldg(p + 2);
        const uint32_t hw[6] = {a.x, a.y, b.x, b.y, c.x, c.y};
#pragma unroll
        for (int t = 0; t < 12; ++t) {
            const uint32_t h = (hw[t >> 1] >> (16 * (t & 1))) & 0xFFFu;
            uint32_t x = (h & 0xFu) | ((h & 0xF0u) << 4) | ((h & 0xF00u) << 8);
            x |= (x & 0x080808u) * 0x1Eu;
            w[t] = x;
        }
    } else {
        const uint4 a = __ldg(wt + 3 * g), b = __ldg(wt + 3 * g + 1), c = __ldg(wt + 3 * g + 2);
        w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
        w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
        w[8] = c.x; w[9] = c.y; w[10] = c.z; w[11] = c.w;
    }
    float2 fbc[4];
#pragma unroll
    for (int c = 0; c < 4; ++c)
        fbc[c] = c0 + c < d.C ? make_float2(e.factor[c0 + c], e.bias[c0 + c]) : make_float2(0.0f, 0.0f);
    // activation folded into the quantizer's clamp
    QParams q0 = e.q0, q1 = e.q1;
    if (ACT == 2) {
        q0.y_hi = fminf(q0.y_hi, 6.0f);
        q1.y_hi = fminf(q1.y_hi, 6.0f);
    }
    const int wp = d.W + 2;
    const int ldi = d.ldi;
    const int per_pass = n_cons / G4;   // strips per pass of the consumers
    griddep_wait();

    int it = 0;
    for (uint32_t u = blockIdx.x; u < static_cast<uint32_t>(d.n_units); u += gridDim.x, ++it) {
        const int stage = it % d.n_stages;
        if (!mbar_wait_warp(bar0 + 8 * stage, static_cast<uint32_t>(it / d.n_stages) & 1u, d.wait_limit)) {
            if ((threadIdx.x & 31) == 0) atomicExch(d.err, ERR_WAIT_FULL);
            break;
        }
        int n0, r0, k;
        size_t off;
        uint32_t bytes;
        dw_unit(d, S, u, n0, r0, k, off, bytes);
        const int nstrip = k * d.R * d.strips;
        const uint8_t* sb = dw_smem + stage * d.stage_bytes + c0;
        for (int sl = static_cast<int>(threadIdx.x) / G4; sl < nstrip; sl += per_pass) {
            const int kk = k == 1 ? 0 : static_cast<int>(fdiv(static_cast<uint32_t>(sl), d.fd_rs));
            const int rem = sl - kk * d.R * d.strips;
            const int rr = static_cast<int>(fdiv(static_cast<uint32_t>(rem), d.fd_strips));
            const int cs = rem - rr * d.strips;
            const uint8_t* base = sb + ((kk * d.rows_img + rr * S) * wp + cs * (T * S)) * ldi;
            int acc[T][4];
#pragma unroll
            for (int t = 0; t < T; ++t)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[t][c] = kRoundMagicBits;   // float-conversion bias (see dequant16)
#pragma unroll
            for (int j = 0; j < S * (T - 1) + 3; ++j) {
                const uint8_t* col = base + j * ldi;
                uint32_t y[4];
                col_transpose3(*reinterpret_cast<const uint32_t*>(col),
                               *reinterpret_cast<const uint32_t*>(col + wp * ldi),
                               *reinterpret_cast<const uint32_t*>(col + 2 * wp * ldi), y);
#pragma unroll
                for (int t = 0; t < T; ++t) {
                    const int jj = j - t * S;   // kernel column of this input column for position t
                    if (jj >= 0 && jj < 3) {
#pragma unroll
                        for (int c = 0; c < 4; ++c)
                            acc[t][c] = __dp4a(static_cast<int>(y[c]), static_cast<int>(w[4 * jj + c]), acc[t][c]);
                    }
                }
            }
            // 16 values = T positions x 4 channels (T < 4: upper values unused)
            uint32_t v[16];
            float2 fb[16];
#pragma unroll
            for (int t = 0; t < 4; ++t)
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    v[4 * t + c] = t < T ? static_cast<uint32_t>(acc[t < T ? t : 0][c]) : kRoundMagicBits;
                    fb[4 * t + c] = fbc[c];
                }
            float y[16];
            dequant16<true>(v, fb, 0, y, false);
            if (ACT != 0) {
#pragma unroll
                for (int j = 0; j < 16; ++j) y[j] = fmaxf(y[j], 0.0f);
            }
            const int n = n0 + kk, oh = r0 + rr, ow = cs * T;
            const size_t pq = (static_cast<size_t>(n) * (d.OH + 2) + oh + 1) * (d.OW + 2) + ow + 1;
            if (e.out_q0) {
                uint32_t q[4];
                quant16q<ACT == 0>(y, q0, e.s0, q);
                int8_t* o = e.out_q0 + pq * e.ldq0 + c0;
#pragma unroll
                for (int t = 0; t < T; ++t) st_u32(o + t * e.ldq0, q[t]);
            }
            if (e.out_q1) {
                uint32_t q[4];
                quant16q<ACT == 0>(y, q1, e.s1, q);
                int8_t* o = e.out_q1 + pq * e.ldq1 + c0;
#pragma unroll
                for (int t = 0; t < T; ++t) st_u32(o + t * e.ldq1, q[t]);
            }
        }
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(bar0 + 8 * (kDwMaxStages + stage));
    }
}

// ------------------------------------------------------------------ stem maxpool

// 3x3/s2/p1 maxpool (padding never wins) of an fp32 map [N][H][W][C]; writes the
// pooled fp32 map and its (bordered) codes.  Quantization is monotone, so pooling the fp32
// values and then quantizing equals the reference's order (ref_e2e.py:192-203).
__global__ void maxpool_kernel(const float* __restrict__ in, int N, int H, int W, int C, int OH, int OW,
                               const EpiParams e) {
    griddep_launch();
    griddep_wait();
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
                m = fmaxf(m, in[f32_off((static_cast<size_t>(n) * H + ih) * W + iw, c, C)]);
            }
        }
        if (e.out_f32) e.out_f32[f32_off(p, c, C)] = m;
        const size_t pq = (static_cast<size_t>(n) * (OH + 2) + oh + 1) * (OW + 2) + ow + 1;
        if (e.out_q0) e.out_q0[pq * e.ldq0 + c] = sat8(quant_code(m, e.inv0, e.s0));
        if (e.out_q1) e.out_q1[pq * e.ldq1 + c] = sat8(quant_code(m, e.inv1, e.s1));
    }
}

// ------------------------------------------------------------------ quantize (test entry)

// codes[i] of x[i] through the same device paths the epilogues use: quant16q
// on full groups of 16, quant_code on the tail.
__global__ void quantize_kernel(const float* __restrict__ x, size_t n, QParams q, float inv, double s,
                                int8_t* __restrict__ out) {
    const size_t g = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
    const size_t base = g * 16;
    if (base >= n) return;
    if (base + 16 <= n) {
        float y[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) y[j] = x[base + j];
        uint32_t w[4];
        quant16q<true>(y, q, s, w);
#pragma unroll
        for (int j = 0; j < 4; ++j) reinterpret_cast<uint32_t*>(out + base)[j] = w[j];
    } else {
        for (size_t i = base; i < n; ++i) out[i] = sat8(quant_code(x[i], inv, s));
    }
}

// ------------------------------------------------------------------ head

// logits[n][o] = fc_b[o] + sum_c fc_w[o][c] * mean_p x[n][p][c]
// One CTA per image: fixed-order fp32 position sums, float64 FC accumulation.
__global__ void head_kernel(const float* __restrict__ x, int HW, int C, const float* __restrict__ fc_w,
                            const float* __restrict__ fc_b, int n_out, float* __restrict__ logits) {
    griddep_launch();
    griddep_wait();
    extern __shared__ float pooled[];
    const int n = blockIdx.x;
    const size_t p0 = static_cast<size_t>(n) * HW;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        float s = 0.0f;
        for (int p = 0; p < HW; ++p) s = __fadd_rn(s, x[f32_off(p0 + p, c, C)]);
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
