// glsl_prelude.h - TEST INFRASTRUCTURE (oracle pin), NOT THE PRODUCT.
//
// Just enough of GLSL 4.60 + GL_NV_cooperative_vector + explicit fp16 arithmetic for
// the reference's bottleneck-transformer compute shaders to compile as C++ and run on
// the host.  glsl_to_cpp.py turns a *.comp.glsl file into a translation unit that
// includes this header; the shader body itself is not edited.
//
// Semantics provided here (everything else is plain C++ with the GLSL meaning):
//  * float16_t = _Float16 (IEEE binary16, round-to-nearest-even conversions);
//    compiled with -fsingle-precision-constant so literals are float as in GLSL.
//  * coopVecMatMulAddNV(out, in, ..., M, K, RowMajor, false, stride):
//      out[r] = fp16( sum_{k<K} float(W[r][k]) * float(in[k]) + float(b[r]) )
//    with an fp32 accumulator in k order and the bias added last.  The extension
//    leaves the precision to the driver; this is the documented model shared by
//    the oracle restatement and the CUDA kernels.
//  * barrier(): workgroup barrier.  A workgroup's invocations run as ucontext
//    coroutines on one host thread; barrier() yields to a round-robin scheduler,
//    so every invocation reaches each barrier before any passes it.
//  * shared variables are per-host-thread (one workgroup at a time per thread).
//  * workgroups run in parallel over OpenMP threads; atomicAdd is a real atomic.
#pragma once
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <ucontext.h>

#include <vector>

extern "C" {
float expf(float);
float tanhf(float);
float sqrtf(float);
}

typedef _Float16 float16_t;

namespace glsl {

struct uvec3 {
    unsigned x, y, z;
};
inline thread_local uvec3 gl_WorkGroupID;
inline thread_local uvec3 gl_LocalInvocationID;
inline thread_local uvec3 gl_GlobalInvocationID;

inline float exp(float x) { return expf(x); }
inline float tanh(float x) { return tanhf(x); }
inline float sqrt(float x) { return sqrtf(x); }
// GLSL max/min: max(x, y) returns y if x < y, otherwise x.
inline float max(float a, float b) { return a < b ? b : a; }
inline float min(float a, float b) { return b < a ? b : a; }
inline int max(int a, int b) { return a < b ? b : a; }
inline int min(int a, int b) { return b < a ? b : a; }

template <class T, int N>
struct coopvecNV {
    T v[N];
    coopvecNV() = default;
    explicit coopvecNV(T s) {
        for (int i = 0; i < N; ++i) v[i] = s;
    }
    T& operator[](int i) {
        if (i < 0 || i >= N) abort();  // reading past a coopvec is undefined in GLSL
        return v[i];
    }
    const T& operator[](int i) const {
        if (i < 0 || i >= N) abort();
        return v[i];
    }
};

enum {
    gl_ComponentTypeFloat16NV = 1,
    gl_CooperativeVectorMatrixLayoutRowMajorNV = 0,
};

template <class T, int N, class B>
inline void coopVecLoadNV(coopvecNV<T, N>& dst, B* buf, int byte_offset) {
    memcpy(dst.v, (const char*)buf + byte_offset, sizeof(T) * N);
}
template <class T, int N, class B>
inline void coopVecStoreNV(const coopvecNV<T, N>& src, B* buf, int byte_offset) {
    memcpy((char*)buf + byte_offset, src.v, sizeof(T) * N);
}

template <int MO, int KI>
inline void coopVecMatMulAddNV(coopvecNV<float16_t, MO>& out, const coopvecNV<float16_t, KI>& in,
                               int /*in_interp*/, const float16_t* mat, int mat_off_bytes,
                               int /*mat_interp*/, const float16_t* bias, int bias_off_bytes,
                               int /*bias_interp*/, int M, int K, int layout, bool transpose,
                               int stride_bytes) {
    if (M > MO || K > KI || layout != gl_CooperativeVectorMatrixLayoutRowMajorNV || transpose) abort();
    const float16_t* W = mat + mat_off_bytes / 2;
    const float16_t* b = bias + bias_off_bytes / 2;
    const int ld = stride_bytes / 2;
    for (int r = 0; r < M; ++r) {
        float acc = 0.0f;
        for (int k = 0; k < K; ++k) acc += (float)W[(size_t)r * ld + k] * (float)in.v[k];
        out.v[r] = (float16_t)(acc + (float)b[r]);
    }
}

inline int atomicAdd(int& mem, int v) { return __atomic_fetch_add(&mem, v, __ATOMIC_RELAXED); }

// ---- workgroup execution ------------------------------------------------------
struct Invocation {
    ucontext_t ctx;
    bool done;
};
inline thread_local ucontext_t t_sched;
inline thread_local Invocation* t_cur = nullptr;
inline thread_local void (*t_fn)() = nullptr;

inline void barrier() { swapcontext(&t_cur->ctx, &t_sched); }

inline void trampoline() {
    t_fn();
    t_cur->done = true;  // uc_link returns to the scheduler
}

inline void set_ids(unsigned g, unsigned i, unsigned L) {
    gl_WorkGroupID = {g, 0, 0};
    gl_LocalInvocationID = {i, 0, 0};
    gl_GlobalInvocationID = {g * L + i, 0, 0};
}

inline void run_group(unsigned g, unsigned L, bool uses_barrier, void (*fn)()) {
    if (!uses_barrier) {
        for (unsigned i = 0; i < L; ++i) {
            set_ids(g, i, L);
            fn();
        }
        return;
    }
    constexpr size_t kStack = 128 * 1024;
    static thread_local std::vector<Invocation> invs;
    static thread_local std::vector<char> stacks;
    if (invs.size() < L) {
        invs.resize(L);
        stacks.resize((size_t)L * kStack);
    }
    t_fn = fn;
    for (unsigned i = 0; i < L; ++i) {
        getcontext(&invs[i].ctx);
        invs[i].ctx.uc_stack.ss_sp = &stacks[(size_t)i * kStack];
        invs[i].ctx.uc_stack.ss_size = kStack;
        invs[i].ctx.uc_link = &t_sched;
        invs[i].done = false;
        makecontext(&invs[i].ctx, (void (*)())trampoline, 0);
    }
    bool pending = true;
    while (pending) {
        pending = false;
        for (unsigned i = 0; i < L; ++i) {
            if (invs[i].done) continue;
            set_ids(g, i, L);
            t_cur = &invs[i];
            swapcontext(&t_sched, &invs[i].ctx);
            if (!invs[i].done) pending = true;
        }
    }
}

// 2-D workgroups (no barrier): group (gx, gy) of a groups_x x groups_y grid, invocation
// (ix, iy) of an Lx x Ly workgroup.
inline void run_groups_2d(int groups_x, int groups_y, int Lx, int Ly, void (*fn)()) {
#pragma omp parallel for schedule(dynamic, 1)
    for (int g = 0; g < groups_x * groups_y; ++g) {
        const unsigned gx = (unsigned)(g % groups_x), gy = (unsigned)(g / groups_x);
        for (unsigned iy = 0; iy < (unsigned)Ly; ++iy)
            for (unsigned ix = 0; ix < (unsigned)Lx; ++ix) {
                gl_WorkGroupID = {gx, gy, 0};
                gl_LocalInvocationID = {ix, iy, 0};
                gl_GlobalInvocationID = {gx * Lx + ix, gy * Ly + iy, 0};
                fn();
            }
    }
}

inline void run_groups(int n_groups, int L, bool uses_barrier, void (*fn)()) {
#pragma omp parallel for schedule(dynamic, 1)
    for (int g = 0; g < n_groups; ++g) run_group((unsigned)g, (unsigned)L, uses_barrier, fn);
}

}  // namespace glsl
