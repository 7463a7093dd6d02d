/*
 * prism_moe.h - C ABI of the B200 (sm_100a) implementation of Prism's bottleneck
 * transformer / MoE stack.
 *
 * The reference dispatches GLSL compute shaders through Vulkan with three storage
 * buffers and an int32 push-constant block per pass:
 *   binding 0  read-only fp16 weight blob      (prism_moe_bench.cpp:105-112)
 *   binding 1  read/write fp16 feature arena   (split2_qkv_attn_d256.comp.glsl:18-19)
 *   binding 2  int32 aux arena (router output) (moe_router.comp.glsl:19-22)
 * Every offset in a push-constant block is an ELEMENT offset (fp16 elements for
 * bindings 0/1, int32 elements for binding 2), and every weight matrix is row-major
 * [out][in].  This header keeps that contract: the per-pass entry points take the
 * same push-constant structs (same field names and order) plus raw DEVICE pointers
 * for the three bindings and a cudaStream_t passed as void*.  Nothing in this file
 * depends on torch or on CUDA headers.
 *
 * Two groups of entry points:
 *  - per-pass drop-ins (prism_attn_window, prism_router, prism_expert, prism_proj_up,
 *    prism_proj_down, prism_dense_block): one call per reference vkCmdDispatch, same
 *    arithmetic, operating on the caller's arenas in place;
 *  - the fast path (prism_stack_*): the whole stack of a prism_stack_desc over a
 *    batch of frames, with weights repacked once into an aligned device arena and
 *    the per-expert dispatch loop replaced by route -> grouped expert GEMM.
 *
 * All calls are stream-ordered on the caller's stream and never synchronise the
 * host, except prism_stack_create (weight upload/repack) and prism_stack_status.
 * Status codes are returned; prism_last_error_string() describes the last failure
 * on the calling thread.
 */
#ifndef PRISM_MOE_H
#define PRISM_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PRISM_ABI_VERSION 1

/* Status codes.  The reference ignores most VkResults and reports a failed
 * pipeline load as VK_NULL_HANDLE (prism_moe_bench.cpp:22,30); this ABI validates
 * every offset and size on the host and returns one of these instead. */
enum prism_status {
    PRISM_OK = 0,
    PRISM_E_ARG = 1,         /* null pointer, bad enum, inconsistent sizes        */
    PRISM_E_ALIGN = 2,       /* pointer/offset alignment the path requires        */
    PRISM_E_RANGE = 3,       /* offset or size outside the buffer / limit         */
    PRISM_E_CUDA = 4,        /* a CUDA runtime/driver call failed                 */
    PRISM_E_TIMEOUT = 5,     /* a bounded device-side wait gave up                */
    PRISM_E_NOMEM = 6,       /* device allocation failed                          */
    PRISM_E_UNSUPPORTED = 7  /* shape the kernels do not implement (e.g. dim 192) */
};

/* ---- push-constant blocks (field order = the GLSL declaration order) ---------- */

/* split2_qkv_attn_d256.comp.glsl:11-16 */
typedef struct prism_attn_params {
    int32_t n_tokens, dim, n_heads, head_dim;
    int32_t spatial_w, spatial_h, window_size;
    int32_t qkv_w, qkv_b, out_w, out_b;
    int32_t input_offset, output_offset;
} prism_attn_params;

/* moe_router.comp.glsl:11-17 */
typedef struct prism_router_params {
    int32_t n_tokens, dim, n_experts;
    int32_t router_w, router_b;
    int32_t input_offset;
    int32_t assignment_offset;
    int32_t count_offset;
} prism_router_params;

/* moe_expert_skip.comp.glsl:13-19 */
typedef struct prism_expert_params {
    int32_t n_tokens, dim;
    int32_t expert_id;
    int32_t w1_offset, b1_offset, w2_offset, b2_offset;
    int32_t input_offset, output_offset;
    int32_t assignment_offset;
} prism_expert_params;

/* pw_project_128to256.comp.glsl:11-15 and pw_project_256to128.comp.glsl:11-15 */
typedef struct prism_proj_params {
    int32_t n_tokens;
    int32_t w_offset, b_offset;
    int32_t input_offset, output_offset;
} prism_proj_params;

/* TransformerPush, prism_scaling_bench.cpp:60-68 (attention_windowed*.comp.glsl) */
typedef struct prism_dense_params {
    int32_t n_tokens, dim, n_heads, head_dim;
    int32_t spatial_w, spatial_h, window_size;
    int32_t qkv_w_offset, qkv_b_offset;
    int32_t out_w_offset, out_b_offset;
    int32_t ffn_w1_offset, ffn_b1_offset;
    int32_t ffn_w2_offset, ffn_b2_offset;
    int32_t input_offset, output_offset;
} prism_dense_params;

/* ---- context --------------------------------------------------------------- */

typedef struct prism_ctx prism_ctx;

/* Replaces the Vulkan instance/device setup of prism_moe_bench.cpp:55-88 and
 * prism::PrismVulkan::Init (prism_vulkan.h:76).  One context per CUDA device;
 * contexts are independent, one context must not be used from two host threads
 * at the same time. */
int prism_create(int device, prism_ctx** out);
int prism_destroy(prism_ctx* ctx);

/* Text of the last error on the calling host thread ("" if none). */
const char* prism_last_error_string(void);
int prism_abi_version(void);

/* ---- per-pass drop-ins (one call = one reference vkCmdDispatch) -------------
 * weights: device pointer to the fp16 blob (binding 0), weight_elems its length
 * features: device pointer to the fp16 arena (binding 1), feature_elems its length
 * aux: device pointer to the int32 arena (binding 2), aux_elems its length
 * stream: cudaStream_t (NULL = legacy default stream)
 * Offsets in the params are bounds-checked against these lengths. */

/* Replaces vkCmdDispatch(split2_qkv_attn_d256, ceil(W/ws)*ceil(H/ws)) at
 * prism_moe_bench.cpp:417-421: out = x + Wo*MHA_window(x) + bo.  dim 128 or 256,
 * head_dim 32, window_size 8. */
int prism_attn_window(prism_ctx* ctx, const prism_attn_params* p,
                      const void* weights, size_t weight_elems,
                      void* features, size_t feature_elems, void* stream);

/* Replaces vkCmdDispatch(moe_router, ceil(T/256)) at prism_moe_bench.cpp:423-426:
 * N-wide logits (256->N), first-max argmax, aux[assignment_offset+t] = e*,
 * atomicAdd(aux[count_offset+e*], 1).  1 <= n_experts <= 256. */
int prism_router(prism_ctx* ctx, const prism_router_params* p,
                 const void* weights, size_t weight_elems,
                 const void* features, size_t feature_elems,
                 int32_t* aux, size_t aux_elems, void* stream);

/* Replaces one vkCmdDispatch(moe_expert_skip) at prism_moe_bench.cpp:428-436:
 * for tokens t with aux[assignment_offset+t] == expert_id,
 * out[t] = x[t] + W2*gelu(W1*x[t] + b1) + b2. Other tokens are not written. */
int prism_expert(prism_ctx* ctx, const prism_expert_params* p,
                 const void* weights, size_t weight_elems,
                 void* features, size_t feature_elems,
                 const int32_t* aux, size_t aux_elems, void* stream);

/* No counterpart in the reference.  Every expert of one MoE pass in one call,
 * without any device allocation: equivalent to calling prism_expert for expert ids
 * p->expert_id .. p->expert_id + n_experts - 1, where expert k uses the weight
 * offsets of p plus (k - p->expert_id) * expert_stride.  For callers that cannot
 * allocate device memory while the pass runs (e.g. a hook inside a host
 * application's frame loop, where cudaMalloc may synchronize the device and stall
 * the frame, or is not allowed after start-up): the routing scratch (counts,
 * offsets, token permutation, tile list) lives in a fixed device array of about
 * 300 KB that every GPU loading the library keeps until the process exits.
 * Limits and rules:
 *  - p->n_tokens <= PRISM_STATIC_MAX_TOKENS, else PRISM_E_RANGE;
 *  - the first call on a device looks up the array's device address (with the
 *    context's device current); make that first call before any stream capture;
 *  - every call reuses the same array, so calls that overlap on the GPU (other
 *    streams, other host threads, other contexts on the same device) race: order
 *    them on one stream. */
#define PRISM_STATIC_MAX_TOKENS 65536
int prism_expert_all_static(prism_ctx* ctx, const prism_expert_params* p,
                            int32_t n_experts, int32_t expert_stride,
                            const void* weights, size_t weight_elems,
                            void* features, size_t feature_elems,
                            const int32_t* aux, size_t aux_elems, void* stream);

/* pw_project_128to256.comp.glsl: out = relu(Wu*x + bu) (prism_moe_bench.cpp:408-412) */
int prism_proj_up(prism_ctx* ctx, const prism_proj_params* p,
                  const void* weights, size_t weight_elems,
                  void* features, size_t feature_elems, void* stream);

/* pw_project_256to128.comp.glsl: out = Wd*x + bd (prism_moe_bench.cpp:441-444) */
int prism_proj_down(prism_ctx* ctx, const prism_proj_params* p,
                    const void* weights, size_t weight_elems,
                    void* features, size_t feature_elems, void* stream);

/* attention_windowed_d256.comp.glsl / attention_windowed.comp.glsl: attention as in
 * prism_attn_window, then a dense FFN of width ffn_hidden.  The FFN output is
 * accumulated in fp16 over ffn_hidden/ffn_chunk partial products, each of which
 * includes b2 (attention_windowed_d256.comp.glsl:145-177): ffn_chunk = 256 gives the
 * "Standard" d256 shader, ffn_chunk = ffn_hidden the unsplit d128 "Baseline"
 * shader (attention_windowed.comp.glsl:151-170). */
int prism_dense_block(prism_ctx* ctx, const prism_dense_params* p,
                      int32_t ffn_hidden, int32_t ffn_chunk,
                      const void* weights, size_t weight_elems,
                      void* features, size_t feature_elems, void* stream);

/* ---- the encoder / decoder around the stack (prism_moe_bench.cpp:386-471) ----------
 * One call = one reference vkCmdDispatch of the named shader, on CHW fp16 feature maps at
 * element offsets of the caller's arena (binding 1), weights at element offsets of the blob
 * (binding 0), with the shader's own push constants in its declaration order:
 *   PRISM_CODEC_ENC_IC   conv3x3_coopvec_9ch        {in_ch, out_ch, w, h, w_off, b_off, in_off, out_off, relu}
 *   PRISM_CODEC_ENC1     strided_conv_coopvec_32ch  {in_ch, out_ch, in_w, in_h, out_w, out_h, w_off, b_off,
 *   PRISM_CODEC_ENC2     strided_conv_split_64ch     in_off, out_off}
 *   PRISM_CODEC_ENC3     strided_conv_split_128ch
 *   PRISM_CODEC_DEC3     dec3_fused                 {out_w, out_h, in_w, in_h, ch, w_off, b_off, in_off,
 *                                                    skip_off, out_off}
 *   PRISM_CODEC_DEC2     dec2_fused                 {out_w, out_h, in_w, in_h, up_ch, skip_ch, w_off, b_off,
 *   PRISM_CODEC_DEC1     dec1_fused                  in_off, skip_off, out_off}
 *   PRISM_CODEC_OUT12    pw_conv_coopvec_32to12     {in_ch, out_ch, w, h, w_off, b_off, in_off, out_off, relu}
 *   PRISM_CODEC_PIXELSHUFFLE pixelshuffle_sigmoid   {render_w, render_h, display_w, display_h, scale,
 *                                                    in_off, out_off}; RGB to `rgb` (binding 2, fp16)
 * The shaders fix their channel counts in code and do not read the channel push constants;
 * neither does this call.  The contractions run on the tensor cores with the shaders' rounding
 * points; the first call of a kind on a context allocates that kind's weight scratch (a repacked,
 * aligned copy made on the stream before each pass, so calls of one context go on one stream).
 * Maps may sit at any element offset; conv3x3_coopvec_9ch, dec2/dec1_fused and pw_conv_coopvec_32to12
 * run a faster form (input rows staged by TMA, output tiles written by TMA) when every map of the
 * call starts 16-byte aligned and its row width is a multiple of 8 pixels (with out_w <= 2 in_w for
 * the decoders), e.g. the 960x540 frame path of prism_inference_b200/codec.py; both forms give the
 * same results.  A bounded device wait that gives up is reported by prism_ctx_status. */
enum prism_codec_kind {
    PRISM_CODEC_ENC_IC = 0, PRISM_CODEC_ENC1 = 1, PRISM_CODEC_ENC2 = 2, PRISM_CODEC_ENC3 = 3,
    PRISM_CODEC_DEC3 = 4, PRISM_CODEC_DEC2 = 5, PRISM_CODEC_DEC1 = 6, PRISM_CODEC_OUT12 = 7,
    PRISM_CODEC_PIXELSHUFFLE = 8
};
int prism_codec_pass(prism_ctx* ctx, int kind, const int32_t* push, int n_push,
                     const void* weights, size_t weight_elems, void* features, size_t feature_elems,
                     void* rgb, size_t rgb_elems, void* stream);

/* Host-synchronising check (and reset) of the context's device error word, set when a bounded
 * wait of a per-pass kernel gives up: PRISM_E_TIMEOUT, else PRISM_OK. */
int prism_ctx_status(prism_ctx* ctx, void* stream);

/* ---- fast path: a whole stack over a batch of frames ------------------------ */

enum prism_block_kind { PRISM_BLOCK_MOE = 0, PRISM_BLOCK_DENSE = 1 };

/* One transformer block: element offsets into the fp16 blob.  The MoE fields follow
 * the bump layout of prism_moe_bench.cpp:164-172 (router [N][dim] + [N], expert e at
 * expert_* + e*expert_stride); the dense fields follow TransformerPush. */
typedef struct prism_block_desc {
    int32_t kind;
    int32_t qkv_w, qkv_b, out_w, out_b;
    int32_t n_experts, router_w, router_b;
    int32_t expert_w1, expert_b1, expert_w2, expert_b2, expert_stride;
    int32_t ffn_hidden, ffn_chunk, ffn_w1, ffn_b1, ffn_w2, ffn_b2;
} prism_block_desc;

/* The stack: optional 128->256 ReLU adapter, n_blocks blocks, optional 256->128
 * adapter (the sequence of prism_moe_bench.cpp:408-444).  Frames are
 * spatial_h x spatial_w tokens, HWC fp16, consecutive in memory. */
typedef struct prism_stack_desc {
    int32_t dim, n_heads, head_dim;
    int32_t spatial_w, spatial_h, window_size;
    int32_t in_dim;          /* == dim, or 128 with the up adapter          */
    int32_t up_w, up_b;      /* pw_project_128to256 weights, -1 if absent   */
    int32_t out_dim;         /* == dim, or 128 with the down adapter        */
    int32_t down_w, down_b;  /* pw_project_256to128 weights, -1 if absent   */
    int32_t n_blocks;
    const prism_block_desc* blocks;
} prism_stack_desc;

typedef struct prism_stack prism_stack;

/* Validates desc against blob_elems, copies the blob (host or device pointer)
 * into an aligned, repacked device arena and allocates the workspace for up to
 * max_frames frames per forward.  Replaces the reference's weight upload
 * (prism_vulkan.cpp:558-577, LoadWeights) for the transformer stack. */
int prism_stack_create(prism_ctx* ctx, const prism_stack_desc* desc,
                       const void* blob, size_t blob_elems, int blob_on_host,
                       int max_frames, prism_stack** out);
int prism_stack_destroy(prism_stack* st);

/* in: device [frames][spatial_h*spatial_w][in_dim] fp16; out: device
 * [frames][T][out_dim] fp16 (must not alias in).  assign (nullable): device int32
 * [n_moe_blocks][frames*T] receives each MoE block's routing.  frames == 0 is a
 * no-op (in and out may then be NULL).  Stream-ordered, no host synchronisation,
 * no allocation: CUDA-graph capturable. */
int prism_stack_forward(prism_stack* st, const void* in, void* out, int frames,
                        int32_t* assign, void* stream);

/* Fast path of one MoE block on the caller's arenas: the reference's per-block dispatch
 * sequence attn (ci -> f_attn), router (f_attn), experts (f_attn -> co)
 * (prism_moe_bench.cpp:414-438) as the fused tcgen05 kernels of prism_stack_forward.  blk is a
 * stack of exactly one MoE block without adapters (prism_stack_create holds its repacked
 * weights), else PRISM_E_ARG.  features_in / features_out: device [frames][T][dim] fp16,
 * typically the caller's feature arena at the pass's input and output offsets (must not
 * overlap).  assign (nullable): device int32 [frames*T], the routing (the router's
 * assignment_offset); counts (nullable): device int32 [n_experts], the tokens each expert
 * received (the router's count_offset; overwritten, where the reference's atomics add to
 * whatever the arena held).  Stream-ordered, no host synchronisation, graph capturable. */
int prism_moe_block(prism_stack* blk, const void* features_in, void* features_out, int frames,
                    int32_t* assign, int32_t* counts, void* stream);

/* Host-buffer inference, the counterpart of PrismVulkan::Infer (prism_vulkan.h:90-91,
 * prism_vulkan.cpp:1007-1040: upload, run, wait, download, return the GPU time).
 * host_in: host [frames][T][in_dim] fp16; host_out: host [frames][T][out_dim] fp16, or
 * NULL to skip the download (as the reference allows).  Synchronous: returns once host_out
 * is written, with the device error word checked as prism_stack_status does.  *gpu_ms
 * (nullable) receives the device time of the forward alone, as the reference returns the
 * inference time without the copies.  Page-locked host memory (cudaHostAlloc,
 * cudaHostRegister) is copied by DMA; pageable memory goes through the driver's staging.
 * The first host-buffer call allocates two device staging slots (input and output for
 * max_frames each) and three internal streams. */
int prism_stack_infer(prism_stack* st, const void* host_in, void* host_out, int frames,
                      float* gpu_ms);

/* Device-buffer inference, the counterpart of PrismVulkan::InferGPU (prism_vulkan.h:88-95,
 * prism_vulkan.cpp:922-1004: the caller's device buffers with BYTE offsets, for a host that
 * already holds the frames on the GPU, e.g. a game hook).  in_buf + in_offset: device
 * [frames][T][in_dim] fp16; out_buf + out_offset: device [frames][T][out_dim] fp16 (must not
 * overlap the input).  Synchronous like the reference (which waits on its fences); *gpu_ms
 * (nullable) receives the device time of the forward alone.  Both addresses 16-byte aligned:
 * the forward reads and writes the caller's buffers directly; otherwise the data is copied
 * through the stack's device staging slot (allocated on first use, as for prism_stack_infer),
 * as the reference copies through its own feature buffer.  The error word is checked as
 * prism_stack_status does. */
int prism_stack_infer_gpu(prism_stack* st, const void* in_buf, size_t in_offset, void* out_buf,
                          size_t out_offset, int frames, float* gpu_ms);

/* Pipelined host-buffer inference for serving loops.  prism_stack_submit enqueues the
 * upload of host_in on an internal copy stream, the forward on `stream` and the download
 * into host_out (nullable) on a second copy stream, and returns at once with a ticket.
 * Submissions alternate between the two staging slots, so the upload of one and the
 * download of the one before overlap the forward in between; ordering between slot uses is
 * kept on the device (events), never by blocking the host.  host_in and host_out must stay
 * untouched until the ticket completes.  prism_stack_wait: with stream == NULL the host
 * blocks until the ticket's download has landed; otherwise `stream` waits for it on the
 * device (pass cudaStreamLegacy for the legacy default stream).  Waiting on a ticket also
 * covers every earlier one.  Same threading rule as prism_stack_forward. */
int prism_stack_submit(prism_stack* st, const void* host_in, void* host_out, int frames,
                       void* stream, int64_t* ticket);
int prism_stack_wait(prism_stack* st, int64_t ticket, void* stream);

/* Host-synchronising check of the device error word the kernels set when a
 * bounded wait gives up (PRISM_E_TIMEOUT) or an invariant fails; clears it. */
int prism_stack_status(prism_stack* st, void* stream);

/* Diagnostic for the failure path (no counterpart in the reference, whose waits are
 * vkWaitForFences with an infinite timeout, prism_moe_bench.cpp:196-206): launches one
 * kernel that leaves expert 0's routing count one token high, as a forward cut short
 * leaves it, and then waits on a device barrier that nothing releases.  The wait gives up
 * after the library's wait limit (2 s) and sets the error word, so the next
 * prism_stack_status returns PRISM_E_TIMEOUT and resets the routing state.  A forward
 * issued in between finds the counts inconsistent, plans no expert work and reports
 * PRISM_E_TIMEOUT/PRISM_E_RANGE through the same status call.  Stream-ordered. */
int prism_stack_inject_stall(prism_stack* st, void* stream);

/* Per-kernel timing (no counterpart in the reference, whose benches time a whole
 * command buffer with timestamp queries, prism_moe_bench.cpp:183-209).  While
 * enabled, prism_stack_forward brackets every launch with CUDA events on the
 * caller's stream.  prism_stack_profile_read synchronises, adds up the elapsed
 * milliseconds and launch counts per kernel kind (enum prism_kernel_kind, n_kinds
 * entries) since the last read, and clears them. */
enum prism_kernel_kind {
    PRISM_K_PROJ_UP = 0, PRISM_K_ATTN = 1, PRISM_K_ROUTER = 2, PRISM_K_ROUTE = 3,
    PRISM_K_EXPERT = 4, PRISM_K_DENSE_FFN = 5, PRISM_K_PROJ_DOWN = 6, PRISM_K_COPY = 7,
    PRISM_K_COUNT = 8
};
int prism_stack_profile(prism_stack* st, int enable);
int prism_stack_profile_read(prism_stack* st, double* ms, int64_t* launches, int n_kinds);

/* Stack options (no counterpart in the reference, whose engine has one dispatch plan).
 * PRISM_OPT_PAIR_ATTENTION (default 1): forwards of dim-256 blocks whose attention has at
 * most half as many 128-row tiles as the GPU has SMs (one 68x120 frame: 68 tiles) split every
 * tile's heads over a cluster of two CTAs, which shortens the serial chain per tile (the
 * batch-1 latency path); 0 keeps one CTA per tile.  Results are bit-identical either way.
 * PRISM_OPT_BUCKET_ROUTING (default 1): the router of a MoE block writes every token into its
 * expert's bucket (one bucket per expert with room for all tokens: max experts x rows int32,
 * allocated at prism_stack_create when that is at most 256 MB) and the grouped expert kernel
 * plans its tiles from the counts, so a MoE block is two launches instead of three; 0, or a
 * stack over the budget, builds the compact permutation with the route kernel.  Results are
 * bit-identical either way (each expert row depends only on its own token).
 * Returns PRISM_E_ARG for an unknown option. */
enum prism_stack_option { PRISM_OPT_PAIR_ATTENTION = 1, PRISM_OPT_BUCKET_ROUTING = 2 };
int prism_stack_set_option(prism_stack* st, int option, int value);

/* Number of kernel launches one prism_stack_forward issues for `frames`. */
int prism_stack_launch_count(const prism_stack* st, int frames);

/* Per-token element count of the stack's frames (spatial_h*spatial_w). */
int prism_stack_tokens_per_frame(const prism_stack* st);

#ifdef __cplusplus
}
#endif
#endif /* PRISM_MOE_H */
