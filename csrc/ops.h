// Host-side launchers of the hand-written sm_100a kernels (raw pointers, explicit strides).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace trida {

using bf16 = __nv_bfloat16;

// ---- normalisation / rope / activation / embedding (elementwise.cu) ----
void rmsnorm_fwd(const bf16* x, int64_t ldx, const bf16* w, bf16* y, int64_t ldy, float* rstd, int M, int D,
                 float eps, cudaStream_t s);
void rmsnorm_bwd(const bf16* dy, int64_t lddy, const bf16* x, int64_t ldx, const bf16* w, const float* rstd,
                 const bf16* dres, int64_t lddres, bf16* dx, int64_t lddx, float* dw, int M, int D, int sm_count,
                 cudaStream_t s);
void qk_norm_rope_fwd(const bf16* qkv, int64_t ldqkv, const bf16* qw, const bf16* kw, const float* cos_t,
                      const float* sin_t, const int* pos, bf16* q, bf16* k, float* rstd, int M, int Hq, int Hkv,
                      int d, int rd, float eps, cudaStream_t s);
void qk_norm_rope_bwd(const bf16* dq, const bf16* dk, const bf16* qkv, int64_t ldqkv, const bf16* qw,
                      const bf16* kw, const float* cos_t, const float* sin_t, const int* pos, const float* rstd,
                      bf16* dqkv, int64_t lddqkv, float* dqw, float* dkw, int M, int Hq, int Hkv, int d, int rd,
                      int sm_count, cudaStream_t s);
void swiglu_fwd(const bf16* gu, int64_t ldgu, bf16* a, int64_t lda, int M, int F, int sm_count, cudaStream_t s);
void swiglu_bwd(const bf16* da, int64_t ldda, const bf16* gu, int64_t ldgu, bf16* dgu, int64_t lddgu, int M,
                int F, int sm_count, cudaStream_t s);
void embed_fwd(const int64_t* ids, const bf16* table, bf16* out, int M, int D, cudaStream_t s);
void embed_bwd(const int64_t* ids, const bf16* dout, float* dtable, int M, int D, cudaStream_t s);

// ---- block-diffusion attention (bd_attention.cu) ----
struct AttnTensors {
  const bf16 *q, *k, *v;
  int64_t q_tok, k_tok, v_tok, q_b, k_b, v_b;
  bf16* o;
  int64_t o_tok, o_b;
  float* lse;
  int B, T, Hq, Hkv, D;
};
void bd_attn_plan(const int4* meta, int B, int T, int flags, uint8_t* cls, int16_t* fwd_list, int* fwd_cnt,
                  int16_t* bwd_list, int* bwd_cnt, cudaStream_t s);
int bd_attn_fwd(const AttnTensors& t, const int4* meta, const int16_t* fwd_list, const int* fwd_cnt, int flags,
                float scale, cudaStream_t s);
int bd_attn_bwd(const AttnTensors& t, const bf16* dout, int64_t do_tok, int64_t do_b, float* dsum, float* dq_acc,
                bf16* dq, int64_t dq_tok, int64_t dq_b, bf16* dk, int64_t dk_tok, int64_t dk_b, bf16* dv,
                int64_t dv_tok, int64_t dv_b, const int4* meta, const int16_t* bwd_list, const int* bwd_cnt,
                int flags, float scale, int sm_count, cudaStream_t s);

// ---- tcgen05 forward (bd_attention_sm100.cu) ----
void bd_attn_lists128(const uint8_t* cls, int B, int T, int16_t* list, int* cnt, int transpose, cudaStream_t s);
int bd_attn_bwd_sm100(const AttnTensors& t, const bf16* dout, int64_t do_tok, int64_t do_b, const float* dsum,
                      float* dq_acc, bf16* dk, int64_t dk_tok, int64_t dk_b, bf16* dv, int64_t dv_tok, int64_t dv_b,
                      const int4* meta, const int16_t* list128t, const int* cnt128t, const uint4* colmask, int flags,
                      float scale, int* err, cudaStream_t s, long long* dbg = nullptr);
void bd_attn_bwd_prep(const AttnTensors& t, const bf16* dout, int64_t do_tok, int64_t do_b, float* dsum, float* dq_acc,
                      cudaStream_t s);
void bd_attn_dq_convert(const float* dq_acc, bf16* dq, int64_t dq_tok, int64_t dq_b, int B, int T, int Hq, int D,
                        int sm_count, cudaStream_t s);
void bd_attn_tile_masks(const int4* meta, const uint8_t* cls, int B, int T, int flags, uint4* rowmask, uint4* colmask,
                        cudaStream_t s);
int bd_attn_fwd_sm100(const AttnTensors& t, const int4* meta, const int16_t* list128, const int* cnt128,
                      const uint4* rowmask, int flags, float scale, int* err, cudaStream_t s, long long* dbg = nullptr);

// ---- cross-entropy rows (cross_entropy.cu) ----
void ce_rows_fwd_bwd(const float* logits, int64_t ld, const int64_t* target, const float* weight, float grad_scale,
                     int n, int V, float* loss, bf16* dlogits, int64_t ldd, cudaStream_t s);

// ---- optimizer (optim.cu) ----
void sumsq_partial(const float* g, int64_t n, float* partial, int nblocks, cudaStream_t s);
void clip_coef(const float* partial, int nblocks, float max_norm, float* norm_out, float* coef_out,
               cudaStream_t s);
void adamw_step(float* master, bf16* param_bf16, const float* grad, float* m, float* v, int64_t n, float lr,
                float beta1, float beta2, float eps, float wd, int step, const float* coef, cudaStream_t s);
void adamw_step_bf16(bf16* param, const float* grad, float* m, float* v, int64_t n, float lr, float beta1,
                     float beta2, float eps, float wd, int step, const float* coef, cudaStream_t s);

}  // namespace trida
