/* yattn_oracle.h -- CPU oracle for the sm_100a attention path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (yllm_b200/, include/)
 * links, loads or calls this code; only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg do, as the checker.
 *
 * Two builds of yattn_oracle.c share this header:
 *   oracle/liboracle.so          every helper restated here ("port")
 *   oracle/_ref/libyattn_ref.so  helpers (softmax, f16_to_f32, f32_to_f16,
 *                                gdn_state_update, l2norm_inplace,
 *                                rmsnorm_gated, rope_*) taken from the
 *                                reference's own matvec.c / platform.c,
 *                                compiled unmodified ("reference")
 * Both export the same orc_* symbols.  The engine's inline attention loops
 * (engine.c) cannot be compiled on their own, so both builds restate them in
 * the reference's operation order.
 */
#ifndef YATTN_ORACLE_H
#define YATTN_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- which build is this (0 = port, 1 = reference helpers linked) ---- */
int orc_build_kind(void);
int orc_max_threads(void);
void orc_set_threads(int n);

/* ---- helpers (platform.c / matvec.c semantics) ---- */
float    orc_f16_to_f32(uint16_t h);                       /* platform.c:316-338 */
uint16_t orc_f32_to_f16(float f);                          /* platform.c:340-379 */
uint64_t orc_yrng(uint64_t* s);                            /* platform.c:411-417 */
void     orc_softmax(float* v, uint32_t n);                /* matvec.c:1023-1031 */
void     orc_rope_inplace(float* v, uint32_t d, uint32_t pos, float theta);       /* matvec.c:890-904 */
void     orc_rope_inplace_qwen(float* v, uint32_t d, uint32_t pos, float theta);  /* matvec.c:907-921 */
void     orc_rope_inplace_mrope(float* v, uint32_t hd, uint32_t n_dims, uint32_t pos, float theta); /* 924-939 */
void     orc_l2norm_inplace(float* v, uint32_t n, float eps);                      /* matvec.c:942-949 */
void     orc_gdn_state_update(float* S, float* out, const float* q, const float* k,
                              const float* v, const float* gate, const float* beta,
                              uint32_t num_k_heads, uint32_t hk, uint32_t n_vheads, uint32_t hv); /* 975-1004 */
void     orc_rmsnorm_gated_f32(float* y, const float* x, const float* w, const float* z,
                               uint32_t n, float eps);     /* matvec.c:1007-1021, DT_F32 weights */
void     orc_f32_to_f16_buf(const float* src, uint16_t* dst, size_t n);
void     orc_conv1d_update(float* state, float* x, const float* w, uint32_t dim, uint32_t kwidth);
void     orc_gdn_inputs(const float* qkv, float* conv_state, const float* conv_w, const float* alpha,
                        const float* beta_in, const float* dt, const float* a, float* q, float* k, float* v,
                        float* gate, float* beta, uint32_t n_seqs, uint32_t T, uint32_t conv_chan,
                        uint32_t kwidth, uint32_t nk, uint32_t hk, uint32_t nv, uint32_t hv, float eps);
int      orc_sess_kv_save(const uint16_t* kv, uint32_t nb, uint32_t kv_dim, uint32_t max_seq, uint32_t pos,
                          const char* path);
int      orc_sess_kv_load(uint16_t* kv, uint32_t nb, uint32_t kv_dim, uint32_t max_seq, const char* path,
                          uint32_t* pos);
void     orc_q4k_block(float* y, const uint8_t* blk);
void     orc_matmul_f16(float* y, const float* x, const uint16_t* w, uint32_t out, uint32_t in);
void     orc_matmul_q4k(float* y, const float* x, const uint8_t* w, uint32_t out, uint32_t in);
void     orc_gemv_q4k(float* y, const uint8_t* w, const float* x, uint32_t out, uint32_t in, uint32_t B);
void     orc_gemv_f16(float* y, const uint16_t* w, const float* x, uint32_t out, uint32_t in, uint32_t B);
void     orc_rope_store(float* q, float* k, const float* v, uint16_t* kcache, uint16_t* vcache,
                        uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t kv_dim, int kind,
                        uint32_t n_dims, uint32_t pos, float theta);
/* matvec.c:152-165 (rmsnorm; fp32 weights, or fp16 bits when w_f16) */
void     orc_rmsnorm(float* y, const float* x, const void* w, uint32_t n, float eps, int w_f16);
/* engine.c:915-934 / 1036-1072: QK-norm of every q and k head, then orc_rope_store */
void     orc_qknorm_rope_store(float* q, float* k, const float* v, uint16_t* kcache, uint16_t* vcache,
                               uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t kv_dim, int kind,
                               uint32_t n_dims, uint32_t pos, float theta, const void* q_w, const void* k_w,
                               int w_f16, float eps);
void     orc_f16_to_f32_buf(const uint16_t* src, float* dst, size_t n);

/* ---- attention loops (engine.c, restated in operation order) ---- */
/* engine.c:1074-1096: one decode step, keys 0..pos, fp16 K/V rows of kv_dim. */
void orc_attn_decode(float* att_out, const float* q, const uint16_t* kcache, const uint16_t* vcache,
                     uint32_t pos, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                     uint32_t kv_dim);
/* engine.c:533-563: B tokens at pos_start.., token bb attends to keys 0..pos_start+bb.
 * q and att_out rows are q_stride floats apart (the engine uses hidden). */
void orc_attn_prefill(float* att_out, const float* q, const uint16_t* kcache, const uint16_t* vcache,
                      uint32_t pos_start, uint32_t B, uint32_t n_heads, uint32_t n_kv_heads,
                      uint32_t head_dim, uint32_t kv_dim, uint32_t q_stride);
/* engine.c:935-960: qwen35 gated attention = decode loop, then out *= sigmoid(gate). */
void orc_attn_decode_gated(float* att_out, const float* q, const float* gate,
                           const uint16_t* kcache, const uint16_t* vcache,
                           uint32_t pos, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                           uint32_t kv_dim);
/* engine.c:723-734 + 935-960: qwen35 prefill runs token by token; token bb at
 * pos_start+bb uses its own q/gate row (stride q_stride). */
void orc_attn_prefill_gated(float* att_out, const float* q, const float* gate,
                            const uint16_t* kcache, const uint16_t* vcache,
                            uint32_t pos_start, uint32_t B, uint32_t n_heads, uint32_t n_kv_heads,
                            uint32_t head_dim, uint32_t kv_dim, uint32_t q_stride);
/* engine.c:831 + 850-852: one GDN token: state update, then (if w && z) the
 * per-v-head rmsnorm_gated epilogue in place on out. */
void orc_gdn_step(float* S, float* out, const float* q, const float* k, const float* v,
                  const float* gate, const float* beta, uint32_t num_k_heads, uint32_t hk,
                  uint32_t n_vheads, uint32_t hv, const float* norm_w, const float* z, float eps);
/* engine.c:723-734: qwen35 prefill is token by token.  q,k: [T][num_k_heads*hk],
 * v,out,z: [T][n_vheads*hv], gate,beta: [T][n_vheads].  Heads are independent,
 * so the oracle runs them in parallel (same arithmetic per head). */
void orc_gdn_prefill(float* S, float* out, const float* q, const float* k, const float* v,
                     const float* gate, const float* beta, uint32_t T, uint32_t num_k_heads,
                     uint32_t hk, uint32_t n_vheads, uint32_t hv,
                     const float* norm_w, const float* z, float eps);

/* ---- seeded inputs (the generator yllm_b200 runs on the GPU, restated) ----
 * Every operation is an IEEE basic op (+ - * / sqrt fma) in a fixed order, so
 * CPU and GPU produce identical bits. */
double   orc_det_log(double x);                 /* x > 0 */
double   orc_det_exp(double x);                 /* |x| < 700 */
void     orc_det_sincos(double x, double* s, double* c);  /* |x| < 2^20 */
uint64_t orc_stream_draw(uint64_t seed, uint64_t k);      /* k-th yrng() output of stream `seed` */
double   orc_normal_d(uint64_t seed, uint64_t i);         /* i-th N(0,1) value (Box-Muller) */
void     orc_fill_normal(uint64_t seed, uint64_t first, size_t n, double scale, float* out);
/* qwen half-split RoPE (pairs j, j+hd/2) on rows of n_heads*hd floats; row r is
 * at position pos0 + r; angles pos * theta^(-2j/hd) in double. */
void     orc_rope_rows(float* x, size_t n_rows, uint32_t n_heads, uint32_t hd,
                       uint32_t pos0, double theta);
void     orc_round_f16(const float* x, size_t n, uint16_t* out);      /* engine f32_to_f16 */
void     orc_round_f16_inplace(float* x, size_t n);                   /* x = f16_to_f32(f32_to_f16(x)) */
void     orc_round_bf16_inplace(float* x, size_t n);                  /* truncate to bf16 */
void     orc_gdn_gates(uint64_t seed_a, uint64_t seed_b, uint64_t first, size_t n,
                       float* gate, float* beta);   /* gate=-softplus(z_a), beta=sigmoid(z_b) */
/* bf16(N(0,1)) rows of n_heads*hd, then l2norm_inplace per head (eps). */
void     orc_gdn_qk(uint64_t seed, uint64_t first_row, size_t n_rows, uint32_t n_heads,
                    uint32_t hd, float eps, float* out);
uint32_t orc_ctx_len(uint64_t seed, uint32_t i, uint32_t lo, uint32_t hi);   /* U[lo,hi] */
uint64_t orc_fnv1a(const void* p, size_t n);
/* FNV-1a 64 over the 64-bit words of each 64 KiB block, then over the block
 * hashes (the definition yattn_checksum uses); n a multiple of 8. */
uint64_t orc_checksum64(const void* p, size_t n);

#ifdef __cplusplus
}
#endif
#endif
