/*
 * prism_oracle.h - TEST INFRASTRUCTURE, NOT THE PRODUCT.
 *
 * Scalar fp32 C++ restatement of the reference's GLSL shaders for the bottleneck
 * transformer / MoE path.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load this library, and only as the checker.
 *
 * Pinning: the reference has no tests, fixtures or golden vectors and cannot run
 * here (Vulkan + VK_NV_cooperative_vector, Win32 host code).  This restatement is
 * pinned against the reference's own shader SOURCES executed on the CPU: the
 * recipe in oracle/glsl_ref/ compiles the unmodified *.comp.glsl files as C++
 * through a documented cooperative-vector shim into oracle/_ref/, and
 * tests/golden/ holds vectors produced that way.  The one assumption both share is
 * the driver-defined coopVecMatMulAddNV arithmetic: fp32 accumulation in k order,
 * bias added last, one round-to-nearest-even to fp16.
 *
 * All buffers are host memory.  fp16 values are passed as uint16_t bit patterns.
 */
#ifndef PRISM_ORACLE_H
#define PRISM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#include "../include/prism_moe.h"

#ifdef __cplusplus
extern "C" {
#endif

/* split2_qkv_attn_d256.comp.glsl:24-79 (dim 256) and attention_windowed.comp.glsl
 * steps 1-3 (dim 128): features[output_offset + t*dim] = x + Wo*MHA_window(x) + bo
 * for every valid token t of the frame. */
void oracle_attn_window(const prism_attn_params* p, const uint16_t* weights,
                        uint16_t* features);

/* N-wide router: moe_ffn_16exp.comp.glsl:27-34 generalised to n_experts, with the
 * argmax / count rule of moe_router.comp.glsl:40-48.  margin (nullable) receives
 * best - second-best logit (fp32 of the fp16 logits; +inf when n_experts == 1). */
void oracle_router(const prism_router_params* p, const uint16_t* weights,
                   const uint16_t* features, int32_t* aux, float* margin);

/* moe_expert_skip.comp.glsl:25-54 */
void oracle_expert(const prism_expert_params* p, const uint16_t* weights,
                   uint16_t* features, const int32_t* aux);

/* pw_project_128to256.comp.glsl:20-40 / pw_project_256to128.comp.glsl:19-33 */
void oracle_proj_up(const prism_proj_params* p, const uint16_t* weights, uint16_t* features);
void oracle_proj_down(const prism_proj_params* p, const uint16_t* weights, uint16_t* features);

/* attention_windowed_d256.comp.glsl:40-182 (ffn_chunk 256) and
 * attention_windowed.comp.glsl:48-176 (ffn_chunk == ffn_hidden). */
void oracle_dense_block(const prism_dense_params* p, int32_t ffn_hidden, int32_t ffn_chunk,
                        const uint16_t* weights, uint16_t* features);

/* Whole stack over `frames` frames (sequence of prism_moe_bench.cpp:408-444 with
 * per-block offsets).  assign_out (nullable): [n_moe_blocks][frames*T].
 * forced (nullable): routing of another implementation, same shape.  Where the
 * oracle's top-2 margin is below tie_thr and forced differs, the oracle follows
 * forced (counted in stats[1]); a difference at margin >= tie_thr is a hard
 * mismatch (stats[2]) and the oracle keeps its own choice.
 * stats (nullable): [0] routed tokens, [1] followed at a tie, [2] hard mismatches,
 * [3] tokens with margin < tie_thr.  Returns 0, or -1 on an invalid descriptor. */
int oracle_stack_forward(const prism_stack_desc* d, const uint16_t* blob, size_t blob_elems,
                         const uint16_t* in, uint16_t* out, int frames,
                         int32_t* assign_out, const int32_t* forced, float tie_thr,
                         int64_t* stats);

/* The encoder / decoder around the stack (prism_moe_bench.cpp:386-471): one pass of the
 * named shader on CHW feature maps, with the shader's push constants in declaration order
 * (n_push of them) and its bindings: weights (binding 0), features (binding 1) and, for
 * ORACLE_PIXELSHUFFLE only, the fp16 RGB output (binding 2).  Returns 0, or -1 for an
 * unknown kind or a push-constant count that does not match the shader. */
enum oracle_codec_kind {
    ORACLE_CONV3X3_9CH = 0,        /* conv3x3_coopvec_9ch.comp.glsl       */
    ORACLE_STRIDED_CONV_32CH = 1,  /* strided_conv_coopvec_32ch.comp.glsl */
    ORACLE_STRIDED_SPLIT_64CH = 2, /* strided_conv_split_64ch.comp.glsl   */
    ORACLE_STRIDED_SPLIT_128CH = 3,/* strided_conv_split_128ch.comp.glsl  */
    ORACLE_DEC3 = 4,               /* dec3_fused.comp.glsl                */
    ORACLE_DEC2 = 5,               /* dec2_fused.comp.glsl                */
    ORACLE_DEC1 = 6,               /* dec1_fused.comp.glsl                */
    ORACLE_PW_32TO12 = 7,          /* pw_conv_coopvec_32to12.comp.glsl    */
    ORACLE_PIXELSHUFFLE = 8        /* pixelshuffle_sigmoid.comp.glsl      */
};
int oracle_codec_pass(int kind, const int32_t* push, int n_push, const uint16_t* weights,
                      uint16_t* features, uint16_t* rgb);

/* helpers exposed for tests */
uint16_t oracle_f2h(float x);
float oracle_h2f(uint16_t h);
float oracle_gelu_h(float x);      /* h(0.5x(1+tanh(0.7978846(x+0.044715x^3)))) */
int oracle_num_threads(void);
void oracle_set_num_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
