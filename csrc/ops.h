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
                      int d, int rd, float eps, int qstride, cudaStream_t s);
void qk_norm_rope_bwd(const bf16* dq, const bf16* dk, const bf16* qkv, int64_t ldqkv, const bf16* qw,
                      const bf16* kw, const float* cos_t, const float* sin_t, const int* pos, const float* rstd,
                      bf16* dqkv, int64_t lddqkv, float* dqw, float* dkw, int M, int Hq, int Hkv, int d, int rd,
                      int qstride, int sm_count, cudaStream_t s);
// sigmoid output gate of the gated attention; gate head h at qkv columns [h*2d + d, h*2d + 2d)
void attn_gate_fwd(const bf16* o, const bf16* qkv, int64_t ldqkv, bf16* y, int M, int Hq, int d, int sm_count,
                   cudaStream_t s);
void attn_gate_bwd(const bf16* dy, const bf16* o, const bf16* qkv, int64_t ldqkv, bf16* d_o, bf16* dqkv,
                   int64_t lddqkv, int M, int Hq, int d, int sm_count, cudaStream_t s);
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
                      float* dq_acc, float* dk_acc, float* dv_acc, bf16* dk, int64_t dk_tok, int64_t dk_b, bf16* dv,
                      int64_t dv_tok, int64_t dv_b, const int4* meta, const int16_t* list128t, const int* cnt128t,
                      const uint4* colmask, int flags, float scale, int* err, cudaStream_t s, long long* dbg);
void bd_attn_bwd_prep(const AttnTensors& t, const bf16* dout, int64_t do_tok, int64_t do_b, float* dsum, float* dq_acc,
                      float* dk_acc, float* dv_acc, int sm_count, cudaStream_t s);
void bd_attn_dq_convert(const float* dq_acc, bf16* dq, int64_t dq_tok, int64_t dq_b, int B, int T, int Hq, int D,
                        int sm_count, cudaStream_t s);
void bd_attn_tile_masks(const int4* meta, const uint8_t* cls, int B, int T, int flags, uint4* rowmask, uint4* colmask,
                        cudaStream_t s);
int bd_attn_fwd_sm100(const AttnTensors& t, const int4* meta, const int16_t* list128, const int* cnt128,
                      const uint4* rowmask, int flags, float scale, int* err, cudaStream_t s, long long* dbg = nullptr);
// head_dim 256 (bd_attention_d256.cu): forward, and backward as a dK / dV kernel (fp32 partials
// added into dk_acc / dv_acc, which must be zeroed) plus a dQ kernel writing bf16 dq directly
int bd_attn_fwd_d256(const AttnTensors& t, const int16_t* list128, const int* cnt128, const uint4* rowmask,
                     const int4* meta, int flags, float scale, int* err, cudaStream_t s);
int bd_attn_bwd_d256(const AttnTensors& t, const bf16* dout, int64_t do_tok, int64_t do_b, const float* dsum,
                     float* dk_acc, float* dv_acc, bf16* dq, int64_t dq_tok, int64_t dq_b, const int16_t* list128t,
                     const int* cnt128t, const uint4* colmask, const int16_t* list128, const int* cnt128,
                     const uint4* rowmask, float scale, int* err, cudaStream_t s);

// ---- self-speculative sampler (sampler.cu) ----
int spec_sample(const float* vals, const int64_t* idx, int kc, const float* temp, const int* topk, const float* topp,
                const int64_t* seed, int64_t* counter, const int* slot, const int* specs, const int* has_specs,
                int* q_idx, float* q_prob, int* out, int B, int blk, int n, cudaStream_t st);

// ---- serving canvas gated-delta step on tensor cores (gdn_canvas_tc.cu) ----
// state cache fp32 [slots, Hv, 128 (k), 128 (v)]; kbuf / ubuf bf16 [B * n, Hv, 128], gbuf fp32 [B * n, Hv]
int gdn_canvas_tc(const bf16* mixed, int64_t ldm, const bf16* ga, const bf16* gb, int64_t ldg, const float* A_log,
                  const float* dt_bias, const float* ssm, const int* slot, bf16* o, bf16* kbuf, bf16* ubuf, float* gbuf,
                  int B, int n, int n_clean, int Hk, int Hv, float scale, int* err, cudaStream_t st,
                  const bf16* z = nullptr, int64_t ldz = 0, const bf16* gnorm_w = nullptr, float eps = 0.f);
int gdn_commit_tc(const bf16* kbuf, const bf16* ubuf, const float* gbuf, float* ssm, const int* slot, const int* adv,
                  int B, int n, int Hv, int* err, cudaStream_t st);

// ---- gated-delta-rule linear attention (gdn.cu) ----
struct GdnParams {
  int B, T, Hk, Hv, dk, dvh;  // dk, dvh: key / value head dims (128)
  int mode;                  // 0 causal, 1 two-stream [x0 ; xt_1..xt_V]
  int L, V, bd;
  int causal_clean, causal_noisy;
  const uint8_t* doc;        // [B, Lc] document starts of the clean stream (or null)
  const bf16* mixed; int64_t ldm;
  const bf16* ga; const bf16* gb; int64_t ldg;
  const float* A_log; const float* dt_bias;
  float scale;
  float* ckpt;               // gdn_state_floats() floats
  bf16* o;
  const bf16* d_o;
  float* dpart;              // gdn_part_floats(): per-CTA partial gradient rows (backward scratch)
  bf16* dv; int64_t lddv;
  float* dinit;              // gdn_state_floats() floats (two-stream backward)
  float* final_state;        // optional [B, Hv, dk, dvh] state after the last clean token
  float* prep;               // gdn_prep_floats(B * T, Hk, Hv) floats of scratch (training kernels)
};
int64_t gdn_state_floats(const GdnParams& p);
int64_t gdn_part_floats(const GdnParams& p);
int gdn_fwd(const GdnParams& p, cudaStream_t s);
// serving: canvas of p.T rows per request from the state cache [slots, Hv, dk, dvh]; commit
// advances the cached state by adv[b] rows of the canvas (both read p.mixed / p.ga / p.gb rows
// b * p.T + j).
// The state cache is thread-native; `prep` holds gdn_prep_floats(B * T, Hk, Hv) floats written by
// gdn_canvas and read again by gdn_commit.
int64_t gdn_prep_floats(int rows, int Hk, int Hv);
int gdn_canvas(const GdnParams& p, float* prep, const float* ssm, const int* slot, int n_clean, cudaStream_t s);
int gdn_commit(const GdnParams& p, const float* prep, float* ssm, const int* slot, const int* adv, cudaStream_t s);
int gdn_bwd(const GdnParams& p, bf16* dmixed, int64_t lddm, bf16* dga, bf16* dgb, int64_t lddg, float* dA_log,
            float* ddt_bias, cudaStream_t s);
// ---- chunked (WY) gated-delta rule on tcgen05 (gdn_chunk.cu) ----
// C: chunk length (64 causal; the diffusion block for the two-stream layout, 16 / 32 / 64).
struct GdnChunkParams {
  int B, T, Hk, Hv;
  int mode, L, V, C, nch;     // nch: clean-stream chunks per row
  int causal_clean, causal_noisy;
  const uint8_t* doc;
  const bf16* mixed; int64_t ldm;
  const bf16* ga; const bf16* gbeta; int64_t ldg;
  const float* A_log; const float* dt_bias;
  float scale;
  bf16* qk;        // [B*T, Hk, 2, 128] normalised q (times scale) / k
  float* gb;       // [B*T, Hv, 2] log-decay, beta
  bf16* wn; bf16* ut; bf16* kt; bf16* u;   // [B*T, Hv, 128] each
  float* gamma;    // [B, Hv, nch]
  bf16* ckpt;      // [B, Hv, nch, 128, 128]
  bf16* o;         // [B*T, Hv*128]
  float* final_state;
  int* err;
};
int gdn_chunk_fwd(const GdnChunkParams& p, cudaStream_t s);
struct GdnChunkBwdParams {
  GdnChunkParams fwd;        // the forward's geometry and saved buffers (o = forward output)
  const bf16* d_o;
  bf16* du0; bf16* du; bf16* qg; bf16* dpe; bf16* dae; bf16* dw; bf16* tt;   // [B*T, Hv, 128] scratch
  bf16* ds0; bf16* dckpt;    // [B, Hv, nch, 128, 128] scratch
  float* sc;                 // [B*T, Hv, 2]
  float* dpart;              // [B*T, Hv, 260]
  bf16* dmixed; int64_t lddm;
  bf16* dga; bf16* dgb; int64_t lddg;
  float* dA_log; float* ddt_bias;   // accumulated (zero them first)
};
int gdn_chunk_bwd(const GdnChunkBwdParams& p, cudaStream_t s);
struct ConvParams {
  int B, T, C, K;
  int mode, L, V, bd;
  const uint8_t* doc;
  const bf16* x; int64_t ldx;
  const bf16* w;
  bf16* y; int64_t ldy;
};
int gdn_conv_fwd(const ConvParams& p, cudaStream_t s);
int gdn_conv_bwd(const ConvParams& p, const bf16* dy, int64_t lddy, float* dpre, bf16* dx, int64_t lddx, float* dw,
                 cudaStream_t s);
int gdn_gnorm_fwd(const bf16* o, const bf16* z, int64_t ldz, const bf16* w, bf16* y, int64_t rows, int H, float eps,
                  cudaStream_t s);
int gdn_gnorm_bwd(const bf16* dy, const bf16* o, const bf16* z, int64_t ldz, const bf16* w, bf16* d_o, bf16* dz,
                  int64_t lddz, float* dw, int64_t rows, int H, float eps, int sm_count, cudaStream_t s);

// ---- serving decode step (serve.cu) ----
int canvas_attention(const bf16* q, const bf16* kc, const bf16* vc, const int* slot, const int* pos, bf16* out,
                     float* work, int B, int blk, int n_clean, int Hq, int Hkv, int D, int maxlen, int max_keys,
                     float scale, cudaStream_t s, const int* ptab = nullptr, int maxpages = 0);
int64_t canvas_work_floats(int B, int blk, int Hq, int D, int max_keys);
// merge of split-K partial rows (unnormalised o, scaled log2 max, sum) into bf16 out [B * blk, Hq, D]
void canvas_combine(const float* po, const float* pm, const float* pl, bf16* out, int B, int nsplit, int Hq, int blk,
                    int D, cudaStream_t s);
// tensor-core canvas attention (canvas_attn_sm100.cu): cache viewed as [cache_rows, Hkv, D] (a paged
// cache's pages * 64 rows, or slots * maxlen); `work` holds canvas_tc_work_floats floats (0: none needed)
int canvas_attention_tc(const bf16* q, const bf16* kc, const bf16* vc, int64_t cache_rows, int n_slots,
                        const int* slot, const int* pos, bf16* out, float* work, int B, int blk, int n_clean, int Hq,
                        int Hkv, int D, int maxlen, int max_keys, float scale, int* err, cudaStream_t s,
                        const int* ptab, int maxpages);
int64_t canvas_tc_work_floats(int B, int blk, int Hq, int Hkv, int D, int max_keys);
void kv_append(const bf16* k, const bf16* v, int64_t ldv, bf16* kc, bf16* vc, const int* slot, const int* pos, int B,
               int blk, int Hkv, int D, int maxlen, cudaStream_t s, const int* ptab = nullptr, int maxpages = 0);
void canvas_conv(const bf16* x, int64_t ldx, const bf16* win, const bf16* w, bf16* y, int64_t ldy, const int* slot,
                 int B, int blk, int C, int K, cudaStream_t s);
void conv_commit(const bf16* x, int64_t ldx, int rows_per, bf16* win, const int* slot, const int* adv, int B, int C,
                 int K, cudaStream_t s);
void argmax_rows(const float* logits, int64_t ld, int rows, int V, int64_t* out, cudaStream_t s);
void conf_argmax_rows(const float* logits, int rows, int rpb, int64_t sb, int64_t ld, int V, int64_t* idx,
                      float* mx, float* sum, cudaStream_t s);

// ---- symmetric peer memory collectives (symm.cu) ----
// bufs / flags: one pointer per rank (this rank's own at index `rank`, peers' IPC-mapped).
int symm_rs_norm_ag(void* const* parts, void* const* gather, unsigned* const* flags, int rank, int world,
                    unsigned* ctr, int D, int64_t row0, int nrows, bf16* xs, const bf16* w, float eps, int* err,
                    int sm_count, cudaStream_t s);
int symm_allreduce_bf16(void* const* bufs, unsigned* const* flags, int rank, int world, unsigned* ctr, unsigned* done,
                        int64_t off, int64_t n, const bf16* residual, bf16* out, int* err, int sm_count,
                        cudaStream_t s);
int symm_rs_sumsq(void* const* bufs, unsigned* const* flags, int rank, int world, unsigned epoch, int64_t shard_off,
                  int64_t shard_len, float scale, float* shard_out, float* partial, int nblocks, int accumulate,
                  int* err, unsigned* done, int close_slot, cudaStream_t s);
int symm_norm_coef(void* const* partials, unsigned* const* flags, int rank, int world, unsigned epoch, int nblocks,
                   float max_norm, float* norm_out, float* coef_out, int* err, cudaStream_t s);
int symm_adamw_ag(void* const* bufs, unsigned* const* flags, int rank, int world, unsigned epoch, int64_t shard_off,
                  int64_t shard_len, const float* grad, float* master, float* m, float* v, float lr, float b1,
                  float b2, float eps, float wd, int step, const float* coef, unsigned* done, int* err, int sm_count,
                  cudaStream_t s);
int symm_gather_bf16(void* const* bufs, int rank, int world, int64_t shard_len, bf16* dst, int blocks, cudaStream_t s);
int symm_barrier(unsigned* const* flags, int rank, int world, unsigned epoch, int slot, int* err, cudaStream_t s);
int symm_ipc_handle(void* ptr, unsigned char* out64);
void* symm_ipc_open(const unsigned char* in64);
void symm_ipc_close(void* p);

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
