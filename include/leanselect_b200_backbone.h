/*
 * leanselect_b200_backbone.h -- fused elementwise kernels of the benchmark's
 * MiniCPM-shaped host model.
 *
 * These entry points are NOT part of the LeanSelect interface and replace no
 * reference function one-for-one: the reference runs these steps as PyTorch
 * elementwise chains inside its backbone (rms_layernorm minicpm.py:772-798,
 * apply_rotary_pos_emb minicpm.py:1034-1069, the SiLU MLP minicpm.py:1082-1146).
 * The benchmark host model uses them around its cuBLAS projections.  Same
 * conventions as leanselect_b200.h (device pointers, bf16 as uint16_t, the
 * caller's stream, LS_* return codes).
 */
#ifndef LEANSELECT_B200_BACKBONE_H_
#define LEANSELECT_B200_BACKBONE_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* out[r] = x[r] * rsqrt(mean(x[r]^2) + eps) * weight; fp32 math, bf16 I/O,
 * hidden a multiple of 8 and at most 8192. */
int ls_bb_rms_norm(const uint16_t* x, const uint16_t* weight, int64_t rows, int32_t hidden,
                   float eps, uint16_t* out, void* stream);

/* Rotary embedding (rotate-half convention) of a fused projection
 * qkv [tokens, (H + 2G) * D]: q [tokens, H, D] and k [tokens, G, D] rotated by
 * angle positions[t] * inv_freq[i] (inv_freq [D/2] fp32, already divided by
 * any LongRoPE factor) with cos/sin scaled by `scaling`; v [tokens, G, D] is
 * copied.  D must be 128. */
int ls_bb_rope_split(const uint16_t* qkv, const int64_t* positions, const float* inv_freq,
                     float scaling, int64_t tokens, int32_t num_heads, int32_t num_kv_heads,
                     int32_t head_dim, uint16_t* q, uint16_t* k, uint16_t* v, void* stream);

/* out[t, i] = silu(gate_up[t, i]) * gate_up[t, I + i] for gate_up [tokens, 2I]. */
int ls_bb_silu_mul(const uint16_t* gate_up, int64_t tokens, int32_t intermediate, uint16_t* out,
                   void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LEANSELECT_B200_BACKBONE_H_ */
