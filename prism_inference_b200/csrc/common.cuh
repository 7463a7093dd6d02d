// common.cuh - sm_100a building blocks shared by the kernels of libprism_moe.so:
// fp16 helpers, mbarriers with bounded waits, TMA (cp.async.bulk.tensor, no
// multicast), tcgen05 MMA / TMEM, and the shared-memory matrix descriptors.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "../../include/prism_moe.h"

#define PRISM_DEV __device__ __forceinline__

namespace prism {

// ---- error word ---------------------------------------------------------------
// Kernels never trap.  A bounded wait that gives up ORs one of these bits into the
// stack's device error word and the kernel winds down; prism_stack_status() turns
// the word into PRISM_E_TIMEOUT / PRISM_E_RANGE on the host.
enum : uint32_t { ERR_TIMEOUT = 1u, ERR_ROUTE = 2u };

// Upper bound of any spin on an mbarrier: 2 s of %globaltimer.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

PRISM_DEV uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// The dynamic shared-memory base rounded up to 1024 bytes by pointer arithmetic on the
// __shared__ array itself: the compiler then knows every pointer derived from it is in the
// shared window and emits shared-memory loads and stores (a base rebuilt from an integer is a
// generic address, and generic accesses go through the slower L1 path).
PRISM_DEV unsigned char* smem_align1k(unsigned char* raw) {
    return raw + ((1024u - (smem_u32(raw) & 1023u)) & 1023u);
}
PRISM_DEV uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// ---- fp16 -----------------------------------------------------------------------
PRISM_DEV float h2f(__half h) { return __half2float(h); }
PRISM_DEV __half f2h(float f) { return __float2half_rn(f); }
PRISM_DEV float rh(float f) { return __half2float(__float2half_rn(f)); }
// two fp32 -> packed f16x2 (lo = a), round to nearest even
PRISM_DEV uint32_t pack_h2(float a, float b) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %2, %1;" : "=r"(r) : "f"(a), "f"(b));
    return r;
}
PRISM_DEV float lo_h2f(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v & 0xffff))); }
PRISM_DEV float hi_h2f(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v >> 16))); }

// GELU(tanh) of moe_expert_skip.comp.glsl:41-44 in fp32, left-to-right as the GLSL
// writes it; tanh from the hardware tanh.approx.f32 (the result is rounded to fp16).
PRISM_DEV float tanh_approx(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// Same expression with the accurate tanhf (used by the per-pass drop-in kernels).
PRISM_DEV float gelu_exact(float x) {
    float c = __fmul_rn(0.044715f, x);
    c = __fmul_rn(c, x);
    c = __fmul_rn(c, x);
    float inner = __fmul_rn(0.7978846f, __fadd_rn(x, c));
    float t = tanhf(inner);
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, t));
}
// Fast path: the same polynomial refactored for FMAs,
// 0.5x(1 + tanh(x(0.7978846 + 0.7978846*0.044715 x^2))) = hx + hx*t with hx = 0.5x.
PRISM_DEV float gelu_f32(float x) {
    const float x2 = x * x;
    const float inner = x * fmaf(0.035677408f, x2, 0.7978846f);
    const float t = tanh_approx(inner);
    const float hx = 0.5f * x;
    return fmaf(hx, t, hx);
}

// ---- packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction for two values, each
// rounded exactly as the scalar instruction would) -----------------------------------------
PRISM_DEV uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
PRISM_DEV void f2_unpack(uint64_t v, float& lo, float& hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
PRISM_DEV uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
PRISM_DEV uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
PRISM_DEV uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
// h(a0 + b0), h(a1 + b1) packed as f16x2 (lo = pair 0), the adds as one f32x2 instruction
PRISM_DEV uint32_t add_pack_h2(float a0, float a1, float b0, float b1) {
    float s0, s1;
    f2_unpack(f2_add(f2_pack(a0, a1), f2_pack(b0, b1)), s0, s1);
    return pack_h2(s0, s1);
}
// gelu_f32 of two values (the same operations in the same order, so the same results)
PRISM_DEV uint64_t gelu_f32x2(uint64_t x) {
    const uint64_t x2 = f2_mul(x, x);
    const uint64_t inner = f2_mul(x, f2_fma(f2_pack(0.035677408f, 0.035677408f), x2, f2_pack(0.7978846f, 0.7978846f)));
    float i0, i1;
    f2_unpack(inner, i0, i1);
    const uint64_t t = f2_pack(tanh_approx(i0), tanh_approx(i1));
    const uint64_t hx = f2_mul(f2_pack(0.5f, 0.5f), x);
    return f2_fma(hx, t, hx);
}

// ---- mbarrier -------------------------------------------------------------------
PRISM_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
PRISM_DEV void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
PRISM_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
PRISM_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
PRISM_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// The spinning part of a bounded wait, out of line: the kernels wait at many places, and
// inlining this loop at each of them costs instruction-cache capacity that the warps
// issuing MMAs and the epilogues need.
static __device__ __noinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity, volatile int* abort) {
    uint64_t t0 = globaltimer();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0) {
            if (*abort) return false;
            if (globaltimer() - t0 > kWaitLimitNs) {
                *abort = 1;
                return false;
            }
        }
    }
}
// Bounded wait.  Returns false (and raises *abort) if the phase did not complete
// within kWaitLimitNs or another role already aborted.
PRISM_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    return mbar_wait_spin(bar, parity, abort);
}
// Bounded wait by a whole warp with a warp-uniform result: a lane whose wait timed
// out raises *abort, which ends every other lane's wait at its next check.
PRISM_DEV bool mbar_wait_w(uint64_t* bar, uint32_t parity, volatile int* abort) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort));
}
// cp.async (non-bulk) completion tracked by an mbarrier: one arrival per thread.
PRISM_DEV void cp_async_mbar_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// 16-byte global -> shared copy; src_bytes = 0 zero-fills the destination.
PRISM_DEV void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
                 : "memory");
}

// cp.async groups of this thread: close the current group / wait until all have landed
PRISM_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
PRISM_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// ---- programmatic dependent launch ------------------------------------------------------
// The stack's kernels are launched so that each may start (and run its prologue: barrier
// init, TMEM allocation, tensor-map prefetch, weight staging) while the previous kernel of
// the stream finishes; every one of them executes grid_dep_wait() before touching anything
// the previous kernels wrote, which returns once those kernels have completed and their
// memory is visible.
PRISM_DEV void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// This CTA no longer needs to delay the next kernel's launch (its remaining work is an epilogue);
// the next kernel still waits for this one to complete before reading its results.
PRISM_DEV void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// generic-proxy shared-memory writes -> visible to the async proxy (TMA, tcgen05)
PRISM_DEV void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---- TMA (no multicast anywhere in this library) ---------------------------------
PRISM_DEV void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}
PRISM_DEV void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
        "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
PRISM_DEV void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                           int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
        "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}
// Store of a box; elements outside the tensor are not written (masked store).
PRISM_DEV void tma_store_4d(const CUtensorMap* map, uint32_t src, int c0, int c1, int c2, int c3) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                     map),
                 "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
                 : "memory");
}
PRISM_DEV void tma_store_3d(const CUtensorMap* map, uint32_t src, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map),
                 "r"(src), "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}
PRISM_DEV void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// until at most N of this thread's committed bulk store groups still read shared memory
template <int N>
PRISM_DEV void tma_store_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
PRISM_DEV void tma_store_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
PRISM_DEV void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ---- tcgen05 / TMEM ------------------------------------------------------------
PRISM_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {  // whole warp
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
PRISM_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
PRISM_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
PRISM_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D(tmem) (+)= A(smem desc) x B(smem desc)^T, kind::f16 (fp16 inputs, fp32 accumulate)
PRISM_DEV void mma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// D(tmem) (+)= A(tmem) x B(smem desc)^T, kind::f16.  A is M=128 rows x K fp16 in TMEM:
// lane = row, two consecutive-K elements per 32-bit column (K=16 -> 8 columns).
PRISM_DEV void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Warp-collective issue.  The whole issuing warp runs the control flow around its
// MMAs (loops, waits, branches) converged, and `elect.sync` picks the lane that
// issues.  Measured on B200: a 128x128x16 MMA issued from a lane that has branched
// away from its warp costs ~128 cycles whenever any branch or wait separates it from
// the next MMA, against 64 cycles of tensor-pipe time when issued converged.
PRISM_DEV void mma_f16_ss_w(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\t"
        "elect.sync r|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
PRISM_DEV void mma_f16_ts_w(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\t"
        "elect.sync r|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
PRISM_DEV void mma_commit_w(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t.reg .b32 r;\n\t"
        "elect.sync r|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
            smem_u32(bar))
        : "memory");
}

// tcgen05.st 32 lanes x 32 bit, 32 consecutive columns from 32 registers per thread
PRISM_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
// tcgen05.st 32 lanes x 32 bit, 16 consecutive columns
PRISM_DEV void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
PRISM_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// mbarrier arrives once every tcgen05 op this thread issued before has completed
PRISM_DEV void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// Instruction descriptor, kind::f16: A = B = fp16, D = fp32, both K-major.
//  [4,6) D format (1 = f32), [7,10) A format (0 = f16), [10,13) B format (0 = f16),
//  [15] A major, [16] B major (0 = K), [17,23) N >> 3, [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Shared-memory matrix descriptor for a K-major operand stored in the canonical
// swizzled layout: rows of `row_bytes` (128 or 64) bytes, 8-row atoms of
// 8*row_bytes bytes stacked along M/N (SBO = 8*row_bytes), the 16-byte chunk index
// within a row XOR-ed with address bits [7,10) (128B) or [7,9) (64B).
//  [0,14) start >> 4, [16,30) LBO >> 4 (ignored for swizzled K-major, 1),
//  [32,46) SBO >> 4, [46,48) version = 1, [49,52) base offset = 0,
//  [61,64) layout: 2 = SWIZZLE_128B, 4 = SWIZZLE_64B.
enum : int { SW128 = 2, SW64 = 4 };
PRISM_DEV uint64_t sdesc(uint32_t saddr, int layout) {
    const uint32_t sbo = layout == SW128 ? 1024u : 512u;
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(sbo >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)layout << 61);
}

// Byte offset of the 16-byte chunk `chunk` of row `row` inside a swizzled K-major
// block whose base is aligned to the swizzle repeat (1024 B / 512 B).
PRISM_DEV uint32_t sw128_off(uint32_t row, uint32_t chunk) {
    return row * 128u + ((chunk ^ (row & 7u)) << 4);
}
// Four 8x8 fp16 tiles from shared memory, transposed: lanes 8i..8i+7 address the eight 16-byte
// rows of tile i; lane t receives elements (2(t%4), t/4) and (2(t%4)+1, t/4) of each tile.
PRISM_DEV void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr)
                 : "memory");
}
// Four 8x8 fp16 tiles to shared memory: lanes 8i..8i+7 address the eight 16-byte rows of tile i;
// lane t supplies elements (t/4, 2(t%4)) and (t/4, 2(t%4)+1) of each tile.
PRISM_DEV void stsm_x4(uint32_t addr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
    asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(r0), "r"(r1),
                 "r"(r2), "r"(r3)
                 : "memory");
}
PRISM_DEV uint32_t sw64_off(uint32_t row, uint32_t chunk) {
    return row * 64u + ((chunk ^ ((row >> 1) & 3u)) << 4);
}

// tcgen05.ld 32 lanes x 32 bit, 16 consecutive columns -> 16 registers per thread
PRISM_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15])
        : "r"(taddr));
}
// 32 consecutive columns -> 32 registers per thread
PRISM_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
PRISM_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 2^x, hardware approximation (the softmax weights are rounded to fp16 afterwards)
PRISM_DEV float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// IEEE fp16x2 addition, round to nearest even: equals h(float(a) + float(b)) per lane
PRISM_DEV uint32_t hadd2_u32(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
// fp32 + bias for 4 lanes at once (bias read as one 16-byte load)
PRISM_DEV float4 ldg_f4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

PRISM_DEV uint32_t elect_one() {  // 1 on exactly one active lane of the warp
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred P;\n\t.reg .b32 rx;\n\t"
        "elect.sync rx|P, %1;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(pred)
        : "r"(0xffffffffu));
    return pred;
}

PRISM_DEV void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- thread-block clusters (distributed shared memory between the CTAs of one cluster) ----
PRISM_DEV uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// the shared::cluster address of the same shared-memory location in CTA `rank` of the cluster
PRISM_DEV uint32_t peer_addr(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
// whole-cluster execution barrier (every thread of every CTA); orders the shared-memory
// writes before it (barrier initialisation) with the other CTAs' accesses after it
PRISM_DEV void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// arrive on an mbarrier of another CTA of the cluster, releasing this thread's prior writes
PRISM_DEV void mbar_arrive_peer(uint32_t bar_cluster) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
// arrive on a peer's mbarrier and raise its expected transaction bytes (the data follows by
// cp.async.bulk into the peer's shared memory, completing on the same barrier)
PRISM_DEV void mbar_expect_tx_peer(uint32_t bar_cluster, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(bar_cluster),
                 "r"(bytes)
                 : "memory");
}
// bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) from this CTA's
// shared memory into a peer CTA's shared memory; completes as transaction bytes on the
// peer's mbarrier
PRISM_DEV void bulk_copy_to_peer(uint32_t dst_cluster, uint32_t src, uint32_t bytes, uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            dst_cluster),
        "r"(src), "r"(bytes), "r"(bar_cluster)
        : "memory");
}
// asynchronous 16-byte store into a peer CTA's shared memory; its completion adds 16 transaction
// bytes to the peer's mbarrier (with release semantics at cluster scope)
PRISM_DEV void st_async_peer(uint32_t dst_cluster, uint32_t x, uint32_t y, uint32_t z, uint32_t w,
                             uint32_t bar_cluster) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                     dst_cluster),
                 "r"(x), "r"(y), "r"(z), "r"(w), "r"(bar_cluster)
                 : "memory");
}
// try_wait with cluster-scope acquire: for barriers that peers arrive on
PRISM_DEV bool mbar_try_wait_cl(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
static __device__ __noinline__ bool mbar_wait_cl_spin(uint64_t* bar, uint32_t parity, volatile int* abort) {
    uint64_t t0 = globaltimer();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait_cl(bar, parity)) return true;
        if ((it & 255u) == 0) {
            if (*abort) return false;
            if (globaltimer() - t0 > kWaitLimitNs) {
                *abort = 1;
                return false;
            }
        }
    }
}
// bounded wait (as mbar_wait) on a barrier that a peer CTA arrives on
PRISM_DEV bool mbar_wait_cl(uint64_t* bar, uint32_t parity, volatile int* abort) {
    if (mbar_try_wait_cl(bar, parity)) return true;
    return mbar_wait_cl_spin(bar, parity, abort);
}

// launch with programmatic dependent launch and thread-block clusters of `cluster` CTAs
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, int cluster,
                                      cudaStream_t s, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace prism
