// prism_oracle.cpp - TEST INFRASTRUCTURE, NOT THE PRODUCT.
//
// Scalar fp32 C++ restatement of the reference GLSL for the bottleneck transformer /
// MoE path (Prism, shaders/*.comp.glsl).  Only tests/, __graft_entry__.smoke() and
// the cpu_baseline leg of bench.py load it, as the checker.  Pinned against the
// reference shader sources executed through oracle/glsl_ref (see prism_oracle.h).
//
// Rounding model (each line names the shader statement it follows):
//  * h(x): fp32 -> fp16 round-to-nearest-even, wherever the GLSL stores float16_t.
//  * MV(W,b,v): coopVecMatMulAddNV = h(sum_k W[r][k]*v[k] + b[r]) with an fp32
//    accumulator, summed in k order, bias added last (driver-defined in the
//    reference; this is the model the GPU kernels are checked against).
//  * attention scores / softmax / PV in fp32 exactly as the shader loops them.
//  * fp16 + fp16 residual adds are h(float(a) + float(b)), which equals IEEE fp16
//    addition because fp32 holds 2*11+2 bits.
// Build: g++ -O3 -fopenmp -ffp-contract=off (no FMA contraction: every multiply and
// add is rounded separately as in the scalar GLSL).

#include "prism_oracle.h"

#include <math.h>
#include <omp.h>
#include <string.h>

#include <algorithm>
#include <vector>

namespace {

float g_h2f[65536];
struct LutInit {
    LutInit() {
        for (int i = 0; i < 65536; ++i) {
            uint16_t b = (uint16_t)i;
            _Float16 h;
            memcpy(&h, &b, 2);
            g_h2f[i] = (float)h;
        }
    }
} g_lut_init;

inline float h2f(uint16_t b) { return g_h2f[b]; }
inline uint16_t f2h(float x) {
    _Float16 h = (_Float16)x;  // RNE
    uint16_t b;
    memcpy(&b, &h, 2);
    return b;
}
inline float rh(float x) { return h2f(f2h(x)); }

// GELU(tanh) as written in moe_expert_skip.comp.glsl:41-44, evaluated left to right
// in fp32:  0.5 * x * (1.0 + tanh(0.7978846 * (x + 0.044715 * x*x*x)))
inline float gelu_f32(float x) {
    float c = 0.044715f * x;
    c = c * x;
    c = c * x;
    float inner = 0.7978846f * (x + c);
    float t = tanhf(inner);
    float hx = 0.5f * x;
    return hx * (1.0f + t);
}

// Y[t][r] = h( sum_k W[r][k] * X[t][k] + b[r] ),  t < nt, r < N.
// X, Y hold fp16 values as float.  W row stride ldw elements.  Summation runs in k
// order per (t, r); the loop vectorises across 16 tokens, which keeps that order.
constexpr int TB = 16;
void mv_tokens(const uint16_t* W, int ldw, const uint16_t* b, int N, int K,
               const float* X, int ldx, int nt, float* Y, int ldy) {
    std::vector<float> xT((size_t)K * TB);
    for (int t0 = 0; t0 < nt; t0 += TB) {
        int tn = std::min(TB, nt - t0);
        for (int k = 0; k < K; ++k)
            for (int t = 0; t < TB; ++t)
                xT[(size_t)k * TB + t] = t < tn ? X[(size_t)(t0 + t) * ldx + k] : 0.0f;
        for (int r = 0; r < N; ++r) {
            float acc[TB];
            for (int t = 0; t < TB; ++t) acc[t] = 0.0f;
            const uint16_t* wr = W + (size_t)r * ldw;
            for (int k = 0; k < K; ++k) {
                float w = h2f(wr[k]);
                const float* xk = &xT[(size_t)k * TB];
                for (int t = 0; t < TB; ++t) acc[t] += w * xk[t];
            }
            float bias = h2f(b[r]);
            for (int t = 0; t < tn; ++t) Y[(size_t)(t0 + t) * ldy + r] = rh(acc[t] + bias);
        }
    }
}

// One 8x8 window: split2_qkv_attn_d256.comp.glsl:25-76 (dim 256, 8 heads) and
// attention_windowed.comp.glsl:53-148 (dim 128, n_heads heads); head_dim 32.
// x: frame base (fp16 values as float, [T][D]); writes y[64][D] and valid[64].
struct AttnShape {
    int D, n_heads, head_dim, W, H, ws, n_tokens;
    float scale;
};

void attn_window(const AttnShape& s, const uint16_t* wts, int qkv_w, int qkv_b, int out_w,
                 int out_b, const float* x, int wi, float* y, bool* valid) {
    const int D = s.D, S = 64;
    std::vector<float> inp((size_t)S * D), Q((size_t)S * D), K((size_t)S * D), V((size_t)S * D),
        ao((size_t)S * D), po((size_t)S * D);
    int wx = (s.W + s.ws - 1) / s.ws;
    int wy = wi / wx, wxx = wi % wx;
    for (int li = 0; li < S; ++li) {
        int ty = li / s.ws, tx = li % s.ws;
        int gy = wy * s.ws + ty, gx = wxx * s.ws + tx;
        valid[li] = gy < s.H && gx < s.W;  // :31
        int gt = gy * s.W + gx;
        for (int c = 0; c < D; ++c) inp[(size_t)li * D + c] = valid[li] ? x[(size_t)gt * D + c] : 0.0f;  // :36-37
    }
    // :40-51  Q, K, V = MV(Wq|Wk|Wv, bq|bk|bv, inp)
    mv_tokens(wts + qkv_w, D, wts + qkv_b, D, D, inp.data(), D, S, Q.data(), D);
    mv_tokens(wts + qkv_w + D * D, D, wts + qkv_b + D, D, D, inp.data(), D, S, K.data(), D);
    mv_tokens(wts + qkv_w + 2 * D * D, D, wts + qkv_b + 2 * D, D, D, inp.data(), D, S, V.data(), D);
    const int wt = std::min(64, s.n_tokens);  // :33  keys = first min(64, n_tokens) slots
    const int hd = s.head_dim;
    for (int h = 0; h < s.n_heads; ++h) {  // :54-69
        int ch = h * hd;
        for (int i = 0; i < S; ++i) {
            float q[32], sc[64], rr[32];
            for (int d = 0; d < hd; ++d) q[d] = Q[(size_t)i * D + ch + d];
            float mx = -1e9f;
            for (int j = 0; j < wt; ++j) {
                float a = 0.0f;
                for (int d = 0; d < hd; ++d) a += q[d] * K[(size_t)j * D + ch + d];
                a *= s.scale;
                sc[j] = a;
                if (a > mx) mx = a;
            }
            float se = 0.0f;
            for (int d = 0; d < hd; ++d) rr[d] = 0.0f;
            for (int j = 0; j < wt; ++j) {
                float w = expf(sc[j] - mx);
                se += w;
                for (int d = 0; d < hd; ++d) rr[d] += w * V[(size_t)j * D + ch + d];
            }
            float iv = 1.0f / std::max(se, 1e-6f);  // :66
            for (int d = 0; d < hd; ++d) ao[(size_t)i * D + ch + d] = rh(rr[d] * iv);  // :67
        }
    }
    // :71-76  po = MV(Wo, bo, ao); y = po + inp (fp16 add)
    mv_tokens(wts + out_w, D, wts + out_b, D, D, ao.data(), D, S, po.data(), D);
    for (size_t i = 0; i < (size_t)S * D; ++i) y[i] = rh(po[i] + inp[i]);
}

void attn_frame(const AttnShape& s, const uint16_t* wts, int qkv_w, int qkv_b, int out_w,
                int out_b, const float* x, float* y_frame) {
    int wx = (s.W + s.ws - 1) / s.ws, wy = (s.H + s.ws - 1) / s.ws;
    int nwin = wx * wy;
#pragma omp parallel
    {
        std::vector<float> y((size_t)64 * s.D);
        bool valid[64];
#pragma omp for schedule(dynamic, 1)
        for (int wi = 0; wi < nwin; ++wi) {
            attn_window(s, wts, qkv_w, qkv_b, out_w, out_b, x, wi, y.data(), valid);
            int wyy = wi / wx, wxx = wi % wx;
            for (int li = 0; li < 64; ++li) {
                if (!valid[li]) continue;  // :78 masked store
                int gy = wyy * s.ws + li / s.ws, gx = wxx * s.ws + li % s.ws;
                int gt = gy * s.W + gx;
                memcpy(&y_frame[(size_t)gt * s.D], &y[(size_t)li * s.D], sizeof(float) * s.D);
            }
        }
    }
}

// Router over nt tokens.  logits = MV(Wr, br, y); strict '>' scan from e = 0
// (moe_router.comp.glsl:40-45, moe_ffn_16exp.comp.glsl:33-34).
void router_tokens(const uint16_t* wts, int rw, int rb, int N, int D, const float* y, int nt,
                   int32_t* best_out, float* margin_out) {
#pragma omp parallel
    {
        std::vector<float> lg((size_t)TB * N);
#pragma omp for schedule(static)
        for (int t0 = 0; t0 < nt; t0 += TB) {
            int tn = std::min(TB, nt - t0);
            mv_tokens(wts + rw, D, wts + rb, N, D, y + (size_t)t0 * D, D, tn, lg.data(), N);
            for (int t = 0; t < tn; ++t) {
                const float* l = &lg[(size_t)t * N];
                int best = 0;
                float bv = l[0];
                for (int e = 1; e < N; ++e)
                    if (l[e] > bv) { bv = l[e]; best = e; }
                float second = -INFINITY;
                for (int e = 0; e < N; ++e)
                    if (e != best && l[e] > second) second = l[e];
                best_out[t0 + t] = best;
                if (margin_out) margin_out[t0 + t] = bv - second;
            }
        }
    }
}

// Expert FFN on a token list: moe_expert_skip.comp.glsl:32-53.
// z = h( MV(W2, b2, gelu_h(MV(W1, b1, y))) + y )
void expert_tokens(const uint16_t* wts, int w1, int b1, int w2, int b2, int D, const float* y,
                   const int* tok, int nt, float* z_out /*indexed by token*/) {
#pragma omp parallel
    {
        std::vector<float> xin((size_t)TB * D), hid((size_t)TB * D), r((size_t)TB * D);
#pragma omp for schedule(static)
        for (int t0 = 0; t0 < nt; t0 += TB) {
            int tn = std::min(TB, nt - t0);
            for (int t = 0; t < tn; ++t)
                memcpy(&xin[(size_t)t * D], &y[(size_t)tok[t0 + t] * D], sizeof(float) * D);
            mv_tokens(wts + w1, D, wts + b1, D, D, xin.data(), D, tn, hid.data(), D);
            for (size_t i = 0; i < (size_t)tn * D; ++i) hid[i] = rh(gelu_f32(hid[i]));
            mv_tokens(wts + w2, D, wts + b2, D, D, hid.data(), D, tn, r.data(), D);
            for (int t = 0; t < tn; ++t)
                for (int c = 0; c < D; ++c)
                    z_out[(size_t)tok[t0 + t] * D + c] = rh(r[(size_t)t * D + c] + xin[(size_t)t * D + c]);
        }
    }
}

// Dense FFN (attention_windowed_d256.comp.glsl:143-177; attention_windowed.comp.glsl:151-170).
// acc = sum over chunks c (fp16 accumulate) of MV(W2[:, c], b2, gelu_h(MV(W1[c], b1[c], y)));
// out = h(acc - (n_chunks-1)*b2 + y)
void dense_ffn_tokens(const uint16_t* wts, int w1, int b1, int w2, int b2, int D, int hidden,
                      int chunk, const float* y, int nt, float* out) {
    const int nch = hidden / chunk;
#pragma omp parallel
    {
        std::vector<float> xin((size_t)TB * D), hid((size_t)TB * chunk), oc((size_t)TB * D),
            acc((size_t)TB * D);
#pragma omp for schedule(static)
        for (int t0 = 0; t0 < nt; t0 += TB) {
            int tn = std::min(TB, nt - t0);
            memcpy(xin.data(), &y[(size_t)t0 * D], sizeof(float) * tn * D);
            std::fill(acc.begin(), acc.end(), 0.0f);
            for (int c = 0; c < nch; ++c) {
                mv_tokens(wts + w1 + (size_t)c * chunk * D, D, wts + b1 + c * chunk, chunk, D,
                          xin.data(), D, tn, hid.data(), chunk);
                for (size_t i = 0; i < (size_t)tn * chunk; ++i) hid[i] = rh(gelu_f32(hid[i]));
                mv_tokens(wts + w2 + c * chunk, hidden, wts + b2, D, chunk, hid.data(), chunk, tn,
                          oc.data(), D);
                for (size_t i = 0; i < (size_t)tn * D; ++i) acc[i] = rh(acc[i] + oc[i]);  // :167-168
            }
            const float corr = (float)(nch - 1);
            for (int t = 0; t < tn; ++t)
                for (int c = 0; c < D; ++c) {
                    float b2v = h2f(wts[b2 + c]);
                    float v = acc[(size_t)t * D + c] - corr * b2v + xin[(size_t)t * D + c];  // :173-176
                    out[(size_t)(t0 + t) * D + c] = rh(v);
                }
        }
    }
}

void proj_tokens(const uint16_t* wts, int w, int b, int N, int K, bool relu, const float* x,
                 int nt, float* y) {
#pragma omp parallel for schedule(static)
    for (int t0 = 0; t0 < nt; t0 += 256) {
        int tn = std::min(256, nt - t0);
        mv_tokens(wts + w, K, wts + b, N, K, x + (size_t)t0 * K, K, tn, y + (size_t)t0 * N, N);
        if (relu)
            for (size_t i = 0; i < (size_t)tn * N; ++i) {
                float v = y[(size_t)t0 * N + i];
                y[(size_t)t0 * N + i] = v < 0.0f ? 0.0f : v;  // pw_project_128to256.comp.glsl:216-219
            }
    }
}

void load_f(const uint16_t* src, size_t n, float* dst) {
    for (size_t i = 0; i < n; ++i) dst[i] = h2f(src[i]);
}
void store_h(const float* src, size_t n, uint16_t* dst) {
    for (size_t i = 0; i < n; ++i) dst[i] = f2h(src[i]);
}

AttnShape attn_shape(int D, int n_heads, int head_dim, int W, int H, int ws, int n_tokens) {
    AttnShape s{D, n_heads, head_dim, W, H, ws, n_tokens, 0.0f};
    // split2_qkv_attn_d256.comp.glsl:62 uses the literal 0.1767766953 (= 1/sqrt(32));
    // attention_windowed.comp.glsl:101 computes 1.0/sqrt(float(head_dim)).
    s.scale = head_dim == 32 ? 0.1767766953f : 1.0f / sqrtf((float)head_dim);
    return s;
}

}  // namespace

extern "C" {

uint16_t oracle_f2h(float x) { return f2h(x); }
float oracle_h2f(uint16_t h) { return h2f(h); }
float oracle_gelu_h(float x) { return rh(gelu_f32(x)); }
int oracle_num_threads(void) { return omp_get_max_threads(); }
void oracle_set_num_threads(int n) { omp_set_num_threads(n); }

void oracle_attn_window(const prism_attn_params* p, const uint16_t* weights, uint16_t* features) {
    const int T = p->spatial_w * p->spatial_h, D = p->dim;
    // split2_qkv_attn_d256 fixes 8 heads x 32 (dim 256); attention_windowed uses n_heads.
    AttnShape s = attn_shape(D, D / 32, 32, p->spatial_w, p->spatial_h, p->window_size, p->n_tokens);
    std::vector<float> x((size_t)T * D), y((size_t)T * D);
    load_f(features + p->input_offset, (size_t)T * D, x.data());
    load_f(features + p->output_offset, (size_t)T * D, y.data());  // untouched rows keep their value
    attn_frame(s, weights, p->qkv_w, p->qkv_b, p->out_w, p->out_b, x.data(), y.data());
    store_h(y.data(), (size_t)T * D, features + p->output_offset);
}

void oracle_router(const prism_router_params* p, const uint16_t* weights, const uint16_t* features,
                   int32_t* aux, float* margin) {
    const int T = p->n_tokens, D = p->dim, N = p->n_experts;
    std::vector<float> y((size_t)T * D);
    load_f(features + p->input_offset, (size_t)T * D, y.data());
    std::vector<int32_t> best(T);
    router_tokens(weights, p->router_w, p->router_b, N, D, y.data(), T, best.data(), margin);
    for (int t = 0; t < T; ++t) {
        aux[p->assignment_offset + t] = best[t];  // moe_router.comp.glsl:47
        aux[p->count_offset + best[t]] += 1;      // :50 atomicAdd
    }
}

void oracle_expert(const prism_expert_params* p, const uint16_t* weights, uint16_t* features,
                   const int32_t* aux) {
    const int T = p->n_tokens, D = p->dim;
    std::vector<int> tok;
    for (int t = 0; t < T; ++t)
        if (aux[p->assignment_offset + t] == p->expert_id) tok.push_back(t);  // :30
    std::vector<float> y((size_t)T * D), z((size_t)T * D);
    load_f(features + p->input_offset, (size_t)T * D, y.data());
    expert_tokens(weights, p->w1_offset, p->b1_offset, p->w2_offset, p->b2_offset, D, y.data(),
                  tok.data(), (int)tok.size(), z.data());
    for (int t : tok)
        for (int c = 0; c < D; ++c) features[p->output_offset + (size_t)t * D + c] = f2h(z[(size_t)t * D + c]);
}

void oracle_proj_up(const prism_proj_params* p, const uint16_t* weights, uint16_t* features) {
    const int T = p->n_tokens;
    std::vector<float> x((size_t)T * 128), y((size_t)T * 256);
    load_f(features + p->input_offset, x.size(), x.data());
    proj_tokens(weights, p->w_offset, p->b_offset, 256, 128, true, x.data(), T, y.data());
    store_h(y.data(), y.size(), features + p->output_offset);
}

void oracle_proj_down(const prism_proj_params* p, const uint16_t* weights, uint16_t* features) {
    const int T = p->n_tokens;
    std::vector<float> x((size_t)T * 256), y((size_t)T * 128);
    load_f(features + p->input_offset, x.size(), x.data());
    proj_tokens(weights, p->w_offset, p->b_offset, 128, 256, false, x.data(), T, y.data());
    store_h(y.data(), y.size(), features + p->output_offset);
}

void oracle_dense_block(const prism_dense_params* p, int32_t ffn_hidden, int32_t ffn_chunk,
                        const uint16_t* weights, uint16_t* features) {
    const int T = p->spatial_w * p->spatial_h, D = p->dim;
    AttnShape s = attn_shape(D, p->n_heads, p->head_dim, p->spatial_w, p->spatial_h,
                             p->window_size, p->n_tokens);
    std::vector<float> x((size_t)T * D), y((size_t)T * D), o((size_t)T * D);
    load_f(features + p->input_offset, x.size(), x.data());
    attn_frame(s, weights, p->qkv_w_offset, p->qkv_b_offset, p->out_w_offset, p->out_b_offset,
               x.data(), y.data());
    dense_ffn_tokens(weights, p->ffn_w1_offset, p->ffn_b1_offset, p->ffn_w2_offset, p->ffn_b2_offset,
                     D, ffn_hidden, ffn_chunk, y.data(), T, o.data());
    store_h(o.data(), o.size(), features + p->output_offset);
}

int oracle_stack_forward(const prism_stack_desc* d, const uint16_t* blob, size_t blob_elems,
                         const uint16_t* in, uint16_t* out, int frames, int32_t* assign_out,
                         const int32_t* forced, float tie_thr, int64_t* stats) {
    (void)blob_elems;
    if (!d || !blob || !in || !out || frames < 0) return -1;
    const int T = d->spatial_w * d->spatial_h, D = d->dim;
    AttnShape s = attn_shape(D, d->n_heads, d->head_dim, d->spatial_w, d->spatial_h, d->window_size, T);
    int64_t st[4] = {0, 0, 0, 0};
    std::vector<float> xin((size_t)T * d->in_dim), cur((size_t)T * D), att((size_t)T * D),
        nxt((size_t)T * D), outf((size_t)T * d->out_dim), margin(T);
    std::vector<int32_t> best(T);
    for (int f = 0; f < frames; ++f) {
        load_f(in + (size_t)f * T * d->in_dim, xin.size(), xin.data());
        if (d->up_w >= 0)
            proj_tokens(blob, d->up_w, d->up_b, D, d->in_dim, true, xin.data(), T, cur.data());
        else
            cur = xin;
        int moe_idx = 0;
        for (int b = 0; b < d->n_blocks; ++b) {
            const prism_block_desc& bd = d->blocks[b];
            attn_frame(s, blob, bd.qkv_w, bd.qkv_b, bd.out_w, bd.out_b, cur.data(), att.data());
            if (bd.kind == PRISM_BLOCK_DENSE) {
                dense_ffn_tokens(blob, bd.ffn_w1, bd.ffn_b1, bd.ffn_w2, bd.ffn_b2, D, bd.ffn_hidden,
                                 bd.ffn_chunk, att.data(), T, nxt.data());
            } else {
                router_tokens(blob, bd.router_w, bd.router_b, bd.n_experts, D, att.data(), T,
                              best.data(), margin.data());
                size_t abase = (size_t)moe_idx * frames * T + (size_t)f * T;
                for (int t = 0; t < T; ++t) {
                    st[0]++;
                    if (margin[t] < tie_thr) st[3]++;
                    if (forced) {
                        int fe = forced[abase + t];
                        if (fe != best[t]) {
                            if (margin[t] < tie_thr && fe >= 0 && fe < bd.n_experts) {
                                best[t] = fe;
                                st[1]++;
                            } else {
                                st[2]++;
                            }
                        }
                    }
                    if (assign_out) assign_out[abase + t] = best[t];
                }
                std::vector<std::vector<int>> lists(bd.n_experts);
                for (int t = 0; t < T; ++t) lists[best[t]].push_back(t);
                for (int e = 0; e < bd.n_experts; ++e) {
                    if (lists[e].empty()) continue;
                    size_t eo = (size_t)e * bd.expert_stride;
                    expert_tokens(blob, (int)(bd.expert_w1 + eo), (int)(bd.expert_b1 + eo),
                                  (int)(bd.expert_w2 + eo), (int)(bd.expert_b2 + eo), D, att.data(),
                                  lists[e].data(), (int)lists[e].size(), nxt.data());
                }
                moe_idx++;
            }
            std::swap(cur, nxt);
        }
        if (d->down_w >= 0) {
            proj_tokens(blob, d->down_w, d->down_b, d->out_dim, D, false, cur.data(), T, outf.data());
            store_h(outf.data(), outf.size(), out + (size_t)f * T * d->out_dim);
        } else {
            store_h(cur.data(), cur.size(), out + (size_t)f * T * D);
        }
    }
    if (stats)
        for (int i = 0; i < 4; ++i) stats[i] = st[i];
    return 0;
}

// ---- encoder / decoder passes (CHW feature maps) ---------------------------------------
// Each follows its shader line by line; MV() is the coopVecMatMulAddNV model above, on one
// gathered input vector.  The shaders fix their channel counts in the code (loop bounds and
// coopvec sizes); their in/out/up/skip-channel push constants are not read, so neither are
// they here.

namespace {

// h( sum_k W[r*ld + k] * v[k] + b[r] ) for r < M, fp32 accumulator in k order, bias last.
void mv_vec(const uint16_t* W, int ld, const uint16_t* b, int M, int K, const float* v, uint16_t* out) {
    for (int r = 0; r < M; ++r) {
        const uint16_t* wr = W + (size_t)r * ld;
        float acc = 0.0f;
        for (int k = 0; k < K; ++k) acc += h2f(wr[k]) * v[k];
        out[r] = f2h(acc + h2f(b[r]));
    }
}

// 3x3 patch of channels [c0, c0 + nc) around (cy, cx), zero outside the map, in the order
// the shaders gather it: channel, then ky, then kx (e.g. strided_conv_split_64ch.comp.glsl:43-55).
void gather3x3(const uint16_t* F, int in_off, int c0, int nc, int in_w, int in_h, int cy, int cx, float* v) {
    const size_t in_px = (size_t)in_w * in_h;
    int p = 0;
    for (int ic = c0; ic < c0 + nc; ++ic)
        for (int ky = -1; ky <= 1; ++ky)
            for (int kx = -1; kx <= 1; ++kx) {
                const int iy = cy + ky, ix = cx + kx;
                v[p++] = (iy >= 0 && iy < in_h && ix >= 0 && ix < in_w)
                             ? h2f(F[in_off + ic * in_px + (size_t)iy * in_w + ix])
                             : 0.0f;
            }
}

inline uint16_t relu_h(uint16_t v) { return h2f(v) < 0.0f ? f2h(0.0f) : v; }  // `if (v < 0) v = 0` on fp16

}  // namespace

int oracle_codec_pass(int kind, const int32_t* push, int n_push, const uint16_t* W, uint16_t* F, uint16_t* rgb) {
    static const int kPush[9] = {9, 10, 10, 10, 10, 11, 11, 9, 7};
    if (kind < 0 || kind > 8 || n_push != kPush[kind]) return -1;
    const int* q = push;
    if (kind == ORACLE_CONV3X3_9CH || kind == ORACLE_PW_32TO12) {
        // conv3x3_coopvec_9ch.comp.glsl:27-59 (3x3, stride 1) / pw_conv_coopvec_32to12.comp.glsl:24-45
        const int w = q[2], h = q[3], wo = q[4], bo = q[5], in_off = q[6], out_off = q[7], relu = q[8];
        const bool conv = kind == ORACLE_CONV3X3_9CH;
        const int in_ch = conv ? 9 : 32, out_ch = conv ? 32 : 12;
        const int px = w * h, K = conv ? in_ch * 9 : in_ch;
#pragma omp parallel for schedule(static)
        for (int idx = 0; idx < px; ++idx) {
            std::vector<float> v(K);
            std::vector<uint16_t> o(out_ch);
            if (kind == ORACLE_CONV3X3_9CH) gather3x3(F, in_off, 0, in_ch, w, h, idx / w, idx % w, v.data());
            else
                for (int c = 0; c < in_ch; ++c) v[c] = h2f(F[in_off + (size_t)c * px + idx]);
            mv_vec(W + wo, K, W + bo, out_ch, K, v.data(), o.data());
            for (int c = 0; c < out_ch; ++c)
                F[out_off + (size_t)c * px + idx] = relu == 1 ? relu_h(o[c]) : o[c];
        }
        return 0;
    }
    if (kind <= ORACLE_STRIDED_SPLIT_128CH) {
        // stride-2 3x3 convs over 32-channel groups of the input
        const int in_w = q[2], in_h = q[3], out_w = q[4], out_h = q[5], wo = q[6], bo = q[7], in_off = q[8],
                  out_off = q[9];
        // 32 -> 64 in one product; 64 -> 128 and 128 -> 128 in 32-channel groups
        const int in_ch = kind == ORACLE_STRIDED_CONV_32CH ? 32 : kind == ORACLE_STRIDED_SPLIT_64CH ? 64 : 128;
        const int out_ch = kind == ORACLE_STRIDED_CONV_32CH ? 64 : 128;
        const int out_px = out_w * out_h;
        const int groups = kind == ORACLE_STRIDED_CONV_32CH ? 1 : in_ch / 32;
        const int Kg = (in_ch / groups) * 9, ld = in_ch * 9;
#pragma omp parallel for schedule(static)
        for (int idx = 0; idx < out_px; ++idx) {
            const int cy = (idx / out_w) * 2, cx = (idx % out_w) * 2;
            std::vector<float> v(Kg);
            std::vector<uint16_t> part(out_ch), acc(out_ch);
            std::vector<float> sum2(out_ch);
            for (int g = 0; g < groups; ++g) {
                gather3x3(F, in_off, g * (in_ch / groups), in_ch / groups, in_w, in_h, cy, cx, v.data());
                mv_vec(W + wo + g * Kg, ld, W + bo, out_ch, Kg, v.data(), part.data());
                for (int c = 0; c < out_ch; ++c) {
                    if (kind == ORACLE_STRIDED_SPLIT_128CH) {
                        // strided_conv_split_128ch.comp.glsl:81-86: fp16 running sum, bias removed per group
                        acc[c] = g == 0 ? part[c] : f2h(h2f(acc[c]) + h2f(part[c]) - h2f(W[bo + c]));
                    } else if (kind == ORACLE_STRIDED_SPLIT_64CH) {
                        // strided_conv_split_64ch.comp.glsl:87-91: fp32 sum of the two products - bias
                        if (g == 0) sum2[c] = h2f(part[c]);
                        else sum2[c] = sum2[c] + h2f(part[c]) - h2f(W[bo + c]);
                    } else {
                        acc[c] = part[c];  // strided_conv_coopvec_32ch.comp.glsl: one product
                    }
                }
            }
            for (int c = 0; c < out_ch; ++c) {
                uint16_t r;
                if (kind == ORACLE_STRIDED_SPLIT_64CH) r = f2h(sum2[c] < 0.0f ? 0.0f : sum2[c]);
                else r = relu_h(acc[c]);
                F[out_off + (size_t)c * out_px + idx] = r;
            }
        }
        return 0;
    }
    if (kind <= ORACLE_DEC1) {
        // dec*_fused.comp.glsl: nearest-neighbour 2x upsample (clamped to the input map) of the
        // deeper map, concatenated with the skip map, then a pointwise product and ReLU
        // up + skip -> out channels: dec3 128 + 128 -> 128, dec2 128 + 64 -> 64, dec1 64 + 32 -> 32
        const int up_ch = kind == ORACLE_DEC1 ? 64 : 128;
        const int skip_ch = kind == ORACLE_DEC3 ? 128 : kind == ORACLE_DEC2 ? 64 : 32, out_ch = skip_ch;
        const int out_w = q[0], out_h = q[1], in_w = q[2], in_h = q[3];
        const int* r = kind == ORACLE_DEC3 ? q + 5 : q + 6;  // dec3 has no up_channels constant
        const int wo = r[0], bo = r[1], in_off = r[2], skip_off = r[3], out_off = r[4];
        const int out_px = out_w * out_h, in_px = in_w * in_h, K = up_ch + skip_ch;
#pragma omp parallel for schedule(static)
        for (int idx = 0; idx < out_px; ++idx) {
            const int iy = std::min((idx / out_w) / 2, in_h - 1), ix = std::min((idx % out_w) / 2, in_w - 1);
            std::vector<float> v(K);
            std::vector<uint16_t> o(out_ch);
            for (int c = 0; c < up_ch; ++c) v[c] = h2f(F[in_off + (size_t)c * in_px + iy * in_w + ix]);
            for (int c = 0; c < skip_ch; ++c) v[up_ch + c] = h2f(F[skip_off + (size_t)c * out_px + idx]);
            mv_vec(W + wo, K, W + bo, out_ch, K, v.data(), o.data());
            for (int c = 0; c < out_ch; ++c) F[out_off + (size_t)c * out_px + idx] = relu_h(o[c]);
        }
        return 0;
    }
    // pixelshuffle_sigmoid.comp.glsl:26-56: display pixel (ox, oy) takes channel
    // c*s*s + (oy%s)*s + ox%s of render pixel (ox/s, oy/s), through 1/(1+exp(-v)) in fp32
    const int rw = q[0], rh_ = q[1], dw = q[2], dh = q[3], sc = q[4], in_off = q[5], out_off = q[6];
    const size_t rpx = (size_t)rw * rh_;
#pragma omp parallel for schedule(static)
    for (int oy = 0; oy < dh; ++oy)
        for (int ox = 0; ox < dw; ++ox)
            for (int c = 0; c < 3; ++c) {
                const int src_ch = c * sc * sc + (oy % sc) * sc + ox % sc;
                const float v = h2f(F[in_off + src_ch * rpx + (size_t)(oy / sc) * rw + ox / sc]);
                rgb[out_off + (size_t)c * dw * dh + (size_t)oy * dw + ox] = f2h(1.0f / (1.0f + expf(-v)));
            }
    return 0;
}

}  // extern "C"
