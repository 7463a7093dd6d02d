// prism_bench.cpp - native C++ caller of libprism_moe.so through include/prism_moe.h alone.
//
// The counterpart of the reference's bench programs (prism_moe_bench.cpp:213-560): it lays
// out a stack in the flat fp16 blob format of export_weights.py (bump allocation, weight then
// bias per layer, export_weights.py:98-121), fills it with seeded N(0, 0.02) weights or reads a
// `.weights` file of exactly that layout, uploads it with prism_stack_create, and times the
// stack with the reference's protocol - warm-up, then timed iterations each bracketed by GPU
// timestamps, reported as mean / median / p90 (prism_moe_bench.cpp:181,196-208):
//   - device-resident frames through prism_stack_forward,
//   - host frames through prism_stack_infer (the reference's Infer: upload, run, download),
//     and the pipelined prism_stack_submit / prism_stack_wait,
//   - one frame as a replayed CUDA graph (batch-1 latency).
// The host-buffer output is checked bit-equal to the device-resident output.  Prints a
// readable summary and one JSON line.  Exit status: 0 ok, 1 failure, 2 usage, 3 no GPU.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "prism_moe.h"

namespace {

struct Config {
    const char* key;
    int dim, n_heads, n_blocks, n_experts, ffn_hidden;
    bool adapters;
    int router_skew;  // experts 0..router_skew-1 get a per-block router bias (load imbalance)
    const char* description;
};

// Per-block router bias of the skewed configuration: ~half of every block's tokens on 4 experts
// for the seeded weights of the Python generator (prism_inference_b200/configs.py).
const float kSkewBias[22] = {0.0777f, 0.0483f, 0.0288f, 0.0324f, 0.0414f, 0.0504f, 0.0521f, 0.0762f,
                             0.0524f, 0.0083f, 0.0784f, 0.0732f, 0.0614f, 0.0054f, 0.0919f, 0.1032f,
                             0.0414f, 0.0485f, 0.1208f, 0.0787f, 0.1102f, 0.0976f};

const Config kConfigs[] = {
    {"moe16x1", 256, 8, 1, 16, 0, false, 0, "1 MoE block, dim 256, 16 experts"},
    {"dense128x4", 128, 4, 4, 0, 128, false, 0, "dense d128 x4, FFN 128"},
    {"dense256x12", 256, 8, 12, 0, 256, true, 0, "dense d256 x12 + adapters, FFN 256"},
    {"moe64x16", 256, 8, 16, 64, 0, true, 0, "MoE 64 experts x16 blocks + adapters"},
    {"moe32x22skew", 256, 8, 22, 32, 0, true, 4, "MoE 32 experts x22 blocks, router skewed to 4 experts"},
};

struct Layout {
    prism_stack_desc d{};
    std::vector<prism_block_desc> blocks;
    int64_t total = 0;

    int32_t bump(int64_t n) {
        const int64_t o = total;
        total += n;
        return (int32_t)o;
    }
};

// The bump order of the Python layout builder: proj_up, then per block qkv, out, router and
// experts (w1, b1, w2, b2 each) or the dense FFN, then proj_down.
Layout build_layout(const Config& c) {
    Layout L;
    const int64_t D = c.dim;
    L.d.dim = c.dim;
    L.d.n_heads = c.n_heads;
    L.d.head_dim = c.dim / c.n_heads;
    L.d.spatial_w = 120;
    L.d.spatial_h = 68;
    L.d.window_size = 8;
    L.d.in_dim = c.adapters ? 128 : c.dim;
    L.d.out_dim = c.adapters ? 128 : c.dim;
    L.d.up_w = L.d.up_b = L.d.down_w = L.d.down_b = -1;
    if (c.adapters) {
        L.d.up_w = L.bump(256 * 128);
        L.d.up_b = L.bump(256);
    }
    for (int i = 0; i < c.n_blocks; ++i) {
        prism_block_desc b{};
        b.kind = c.n_experts > 0 ? PRISM_BLOCK_MOE : PRISM_BLOCK_DENSE;
        // offsets of the parts a block does not have stay -1 (absent)
        b.router_w = b.router_b = b.expert_w1 = b.expert_b1 = b.expert_w2 = b.expert_b2 = -1;
        b.ffn_w1 = b.ffn_b1 = b.ffn_w2 = b.ffn_b2 = -1;
        b.qkv_w = L.bump(3 * D * D);
        b.qkv_b = L.bump(3 * D);
        b.out_w = L.bump(D * D);
        b.out_b = L.bump(D);
        if (c.n_experts > 0) {
            b.n_experts = c.n_experts;
            b.router_w = L.bump(c.n_experts * D);
            b.router_b = L.bump(c.n_experts);
            b.expert_stride = (int32_t)(2 * D * D + 2 * D);
            for (int e = 0; e < c.n_experts; ++e) {
                const int32_t w1 = L.bump(D * D), b1 = L.bump(D), w2 = L.bump(D * D), b2 = L.bump(D);
                if (e == 0) {
                    b.expert_w1 = w1;
                    b.expert_b1 = b1;
                    b.expert_w2 = w2;
                    b.expert_b2 = b2;
                }
            }
        } else {
            b.ffn_hidden = b.ffn_chunk = c.ffn_hidden;
            b.ffn_w1 = L.bump((int64_t)c.ffn_hidden * D);
            b.ffn_b1 = L.bump(c.ffn_hidden);
            b.ffn_w2 = L.bump(D * c.ffn_hidden);
            b.ffn_b2 = L.bump(D);
        }
        L.blocks.push_back(b);
    }
    if (c.adapters) {
        L.d.down_w = L.bump(128 * 256);
        L.d.down_b = L.bump(128);
    }
    L.d.n_blocks = c.n_blocks;
    L.d.blocks = L.blocks.data();
    return L;
}

// IEEE binary32 -> binary16, round to nearest even (overflow to infinity).
uint16_t to_half(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const int32_t e8 = (int32_t)((x >> 23) & 0xff);
    uint32_t mant = x & 0x7fffffu;
    if (e8 == 0xff) return (uint16_t)(sign | 0x7c00u | (mant ? 0x200u : 0u));
    const int32_t e = e8 - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        const int shift = 14 - e;
        uint32_t h = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) ++h;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;  // a carry rounds up into the exponent
    return (uint16_t)(sign | h);
}

float from_half(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ffu;
    float v;
    if (e == 0) v = std::ldexp((float)m, -24);
    else if (e == 31) v = m ? NAN : INFINITY;
    else v = std::ldexp((float)(m | 0x400u), (int)e - 25);
    uint32_t x;
    std::memcpy(&x, &v, 4);
    x |= sign;
    std::memcpy(&v, &x, 4);
    return v;
}

void fill_normal(uint16_t* p, size_t n, uint64_t seed, float std) {
    std::mt19937_64 rng(seed);
    std::normal_distribution<float> dist(0.0f, std);
    for (size_t i = 0; i < n; ++i) p[i] = to_half(dist(rng));
}

struct Stats {
    double mean, median, p90;
};

Stats stats(std::vector<float> v) {
    std::sort(v.begin(), v.end());
    double s = 0;
    for (float x : v) s += x;
    const size_t n = v.size();
    return {s / n, n % 2 ? v[n / 2] : 0.5 * (v[n / 2 - 1] + v[n / 2]), v[std::min(n - 1, (size_t)std::ceil(0.9 * n) - 1)]};
}

// The layout as JSON (offsets in fp16 elements), for comparison with the Python builder.
void print_layout(const Layout& L) {
    const prism_stack_desc& d = L.d;
    std::printf("{\"total\": %lld, \"in_dim\": %d, \"out_dim\": %d, \"up\": [%d, %d], \"down\": [%d, %d], \"blocks\": [",
                (long long)L.total, d.in_dim, d.out_dim, d.up_w, d.up_b, d.down_w, d.down_b);
    for (size_t i = 0; i < L.blocks.size(); ++i) {
        const prism_block_desc& b = L.blocks[i];
        std::printf("%s[%d, %d, %d, %d, %d, %d, %d, %d, %d, %d, %d, %d, %d, %d, %d, %d, %d, %d, %d]", i ? ", " : "",
                    b.kind, b.qkv_w, b.qkv_b, b.out_w, b.out_b, b.n_experts, b.router_w, b.router_b, b.expert_w1,
                    b.expert_b1, b.expert_w2, b.expert_b2, b.expert_stride, b.ffn_hidden, b.ffn_chunk, b.ffn_w1,
                    b.ffn_b1, b.ffn_w2, b.ffn_b2);
    }
    std::printf("]}\n");
}

int usage() {
    std::fprintf(stderr,
                 "usage: prism_bench [--config KEY] [--frames B] [--warmup W] [--iters K] [--device N]\n"
                 "                   [--weights FILE] [--layout]\n"
                 "  KEY: moe64x16 (default), moe32x22skew, moe16x1, dense256x12, dense128x4\n"
                 "  FILE: raw fp16 blob in the layout of KEY (export_weights.py format)\n"
                 "  --layout: print the blob layout of KEY as JSON and exit (no GPU needed)\n");
    return 2;
}

#define CK(call)                                                                              \
    do {                                                                                      \
        cudaError_t e_ = (call);                                                              \
        if (e_ != cudaSuccess) {                                                              \
            std::fprintf(stderr, "prism_bench: %s failed: %s\n", #call, cudaGetErrorString(e_)); \
            return 1;                                                                         \
        }                                                                                     \
    } while (0)
#define PK(call)                                                                                  \
    do {                                                                                          \
        int r_ = (call);                                                                          \
        if (r_ != PRISM_OK) {                                                                     \
            std::fprintf(stderr, "prism_bench: %s -> %d: %s\n", #call, r_, prism_last_error_string()); \
            return 1;                                                                             \
        }                                                                                         \
    } while (0)

int run(const Config& cfg, int frames, int warmup, int iters, const char* weights, prism_ctx* ctx) {
    Layout L = build_layout(cfg);
    const int64_t T = (int64_t)L.d.spatial_w * L.d.spatial_h;
    const size_t in_elems = (size_t)frames * T * L.d.in_dim, out_elems = (size_t)frames * T * L.d.out_dim;

    // ---- weights: a file of exactly this layout, or seeded synthetic ones
    std::vector<uint16_t> blob((size_t)L.total);
    if (weights) {
        FILE* f = std::fopen(weights, "rb");
        if (!f) {
            std::fprintf(stderr, "prism_bench: cannot open %s\n", weights);
            return 1;
        }
        const size_t got = std::fread(blob.data(), 2, blob.size(), f);
        const bool longer = std::fgetc(f) != EOF;
        std::fclose(f);
        if (got != blob.size() || longer) {
            std::fprintf(stderr, "prism_bench: %s does not hold %lld fp16 values (layout of %s)\n", weights,
                         (long long)L.total, cfg.key);
            return 1;
        }
    } else {
        fill_normal(blob.data(), blob.size(), 0x5EED0000ull, 0.02f);
        if (cfg.router_skew > 0)
            for (int i = 0; i < cfg.n_blocks; ++i)
                for (int e = 0; e < cfg.router_skew; ++e) {
                    uint16_t& h = blob[(size_t)L.blocks[i].router_b + e];
                    h = to_half(from_half(h) + kSkewBias[i % 22]);
                }
    }
    prism_stack* st = nullptr;
    PK(prism_stack_create(ctx, &L.d, blob.data(), blob.size(), 1, frames, &st));

    // ---- frames ~ N(0, 1): page-locked host copy and a device copy
    uint16_t *x_h = nullptr, *y_h = nullptr, *y_ref = nullptr;
    void *x_d = nullptr, *y_d = nullptr;
    CK(cudaHostAlloc((void**)&x_h, in_elems * 2, cudaHostAllocDefault));
    CK(cudaHostAlloc((void**)&y_h, out_elems * 2, cudaHostAllocDefault));
    CK(cudaHostAlloc((void**)&y_ref, out_elems * 2, cudaHostAllocDefault));
    fill_normal(x_h, in_elems, 0x5EEDull, 1.0f);
    CK(cudaMalloc(&x_d, in_elems * 2));
    CK(cudaMalloc(&y_d, out_elems * 2));
    CK(cudaMemcpy(x_d, x_h, in_elems * 2, cudaMemcpyHostToDevice));
    cudaStream_t s;
    CK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    std::vector<cudaEvent_t> ev(iters + 1);
    for (auto& e : ev) CK(cudaEventCreate(&e));
    const double tokens = (double)frames * T;

    // ---- device-resident frames
    for (int i = 0; i < warmup; ++i) PK(prism_stack_forward(st, x_d, y_d, frames, nullptr, s));
    CK(cudaStreamSynchronize(s));
    PK(prism_stack_status(st, s));
    CK(cudaEventRecord(ev[0], s));
    for (int i = 0; i < iters; ++i) {
        PK(prism_stack_forward(st, x_d, y_d, frames, nullptr, s));
        CK(cudaEventRecord(ev[i + 1], s));
    }
    CK(cudaStreamSynchronize(s));
    PK(prism_stack_status(st, s));
    std::vector<float> t_dev(iters);
    for (int i = 0; i < iters; ++i) CK(cudaEventElapsedTime(&t_dev[i], ev[i], ev[i + 1]));
    CK(cudaMemcpy(y_ref, y_d, out_elems * 2, cudaMemcpyDeviceToHost));
    const Stats sd = stats(t_dev);

    // ---- host frames, synchronous (the reference's Infer): GPU time of the forward, and the
    // host's time of the whole call (upload, forward, download)
    std::vector<float> t_inf(iters), t_call(iters);
    for (int i = 0; i < warmup; ++i) PK(prism_stack_infer(st, x_h, y_h, frames, nullptr));
    for (int i = 0; i < iters; ++i) {
        const auto c0 = std::chrono::steady_clock::now();
        PK(prism_stack_infer(st, x_h, y_h, frames, &t_inf[i]));
        t_call[i] = std::chrono::duration<float, std::milli>(std::chrono::steady_clock::now() - c0).count();
    }
    if (std::memcmp(y_h, y_ref, out_elems * 2) != 0) {
        std::fprintf(stderr, "prism_bench: prism_stack_infer output differs from prism_stack_forward's\n");
        return 1;
    }
    const Stats si = stats(t_inf), sc = stats(t_call);

    // ---- host frames, pipelined: GPU time from the first submission to the last download
    int64_t ticket = 0;
    for (int i = 0; i < warmup; ++i) PK(prism_stack_submit(st, x_h, y_h, frames, s, &ticket));
    PK(prism_stack_wait(st, ticket, nullptr));
    std::memset(y_h, 0, out_elems * 2);
    CK(cudaEventRecord(ev[0], s));
    CK(cudaEventSynchronize(ev[0]));
    for (int i = 0; i < iters; ++i) PK(prism_stack_submit(st, x_h, y_h, frames, s, &ticket));
    PK(prism_stack_wait(st, ticket, s));
    CK(cudaEventRecord(ev[1], s));
    CK(cudaStreamSynchronize(s));
    PK(prism_stack_status(st, s));
    float t_pipe = 0;
    CK(cudaEventElapsedTime(&t_pipe, ev[0], ev[1]));
    t_pipe /= iters;
    if (std::memcmp(y_h, y_ref, out_elems * 2) != 0) {
        std::fprintf(stderr, "prism_bench: prism_stack_submit output differs from prism_stack_forward's\n");
        return 1;
    }

    // ---- batch 1: one frame through the whole stack as a replayed CUDA graph
    cudaGraph_t graph;
    cudaGraphExec_t exec;
    CK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    PK(prism_stack_forward(st, x_d, y_d, 1, nullptr, s));
    CK(cudaStreamEndCapture(s, &graph));
    CK(cudaGraphInstantiate(&exec, graph, 0));
    for (int i = 0; i < warmup; ++i) CK(cudaGraphLaunch(exec, s));
    CK(cudaEventRecord(ev[0], s));
    for (int i = 0; i < iters; ++i) {
        CK(cudaGraphLaunch(exec, s));
        CK(cudaEventRecord(ev[i + 1], s));
    }
    CK(cudaStreamSynchronize(s));
    PK(prism_stack_status(st, s));
    std::vector<float> t_b1(iters);
    for (int i = 0; i < iters; ++i) CK(cudaEventElapsedTime(&t_b1[i], ev[i], ev[i + 1]));
    const Stats s1 = stats(t_b1);
    CK(cudaGraphExecDestroy(exec));
    CK(cudaGraphDestroy(graph));

    std::printf("prism_bench: %s (%s), %d frames of %lldx%lld tokens, %d warm-up + %d timed iterations\n",
                cfg.key, cfg.description, frames, (long long)L.d.spatial_h, (long long)L.d.spatial_w, warmup,
                iters);
    std::printf("  device buffers   %8.3f ms/step mean, %8.3f median, %8.3f p90  -> %.3f M tokens/s, %.1f frames/s\n",
                sd.mean, sd.median, sd.p90, tokens / sd.mean / 1e3, frames / sd.mean * 1e3);
    std::printf("  infer (host)     %8.3f ms GPU mean, %8.3f ms per call (upload + forward + download)\n", si.mean,
                sc.mean);
    std::printf("  submit/wait      %8.3f ms/step -> %.3f M tokens/s with host copies overlapped\n", t_pipe,
                tokens / t_pipe / 1e3);
    std::printf("  batch 1 (graph)  %8.3f ms mean, %8.3f median, %8.3f p90\n", s1.mean, s1.median, s1.p90);
    std::printf(
        "{\"config\": \"%s\", \"frames\": %d, \"tokens_per_frame\": %lld, \"warmup\": %d, \"iters\": %d, "
        "\"weights\": \"%s\", \"device_ms\": {\"mean\": %.4f, \"median\": %.4f, \"p90\": %.4f}, "
        "\"device_tokens_per_s\": %.1f, \"infer_gpu_ms\": %.4f, \"infer_call_ms\": %.4f, "
        "\"pipelined_ms\": %.4f, \"pipelined_tokens_per_s\": %.1f, "
        "\"batch1_ms\": {\"mean\": %.4f, \"median\": %.4f, \"p90\": %.4f}}\n",
        cfg.key, frames, (long long)T, warmup, iters, weights ? "file" : "synthetic", sd.mean, sd.median, sd.p90,
        tokens / sd.mean * 1e3, si.mean, sc.mean, t_pipe, tokens / t_pipe * 1e3, s1.mean, s1.median, s1.p90);

    for (auto& e : ev) cudaEventDestroy(e);
    cudaStreamDestroy(s);
    cudaFree(x_d);
    cudaFree(y_d);
    cudaFreeHost(x_h);
    cudaFreeHost(y_h);
    cudaFreeHost(y_ref);
    PK(prism_stack_destroy(st));
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    const char* key = "moe64x16";
    const char* weights = nullptr;
    int frames = 64, warmup = 10, iters = 100, device = 0;
    bool layout_only = false;
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        if (a == "--help" || a == "-h") {
            usage();
            return 0;
        }
        if (a == "--layout") {
            layout_only = true;
            continue;
        }
        if (i + 1 >= argc) return usage();
        const char* v = argv[++i];
        if (a == "--config") key = v;
        else if (a == "--frames") frames = std::atoi(v);
        else if (a == "--warmup") warmup = std::atoi(v);
        else if (a == "--iters") iters = std::atoi(v);
        else if (a == "--device") device = std::atoi(v);
        else if (a == "--weights") weights = v;
        else return usage();
    }
    const Config* cfg = nullptr;
    for (const Config& c : kConfigs)
        if (std::strcmp(c.key, key) == 0) cfg = &c;
    if (!cfg || frames < 1 || warmup < 0 || iters < 1) return usage();
    if (layout_only) {
        print_layout(build_layout(*cfg));
        return 0;
    }
    prism_ctx* ctx = nullptr;
    if (prism_create(device, &ctx) != PRISM_OK) {
        std::fprintf(stderr, "prism_bench: no usable CUDA device %d: %s\n", device, prism_last_error_string());
        return 3;
    }
    const int rc = run(*cfg, frames, warmup, iters, weights, ctx);
    prism_destroy(ctx);
    return rc;
}
