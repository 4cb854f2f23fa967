/* yattn_oracle.c -- CPU oracle for the sm_100a attention path (TEST INFRASTRUCTURE).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
 * file, as the checker.  The product (yllm_b200/) never links or calls it.
 *
 * Build with the reference's own flags (Makefile:122,165):
 *   -O2 -std=c99 -mavx2 -mfma -mf16c -fopenmp
 * In ISO C mode gcc does not contract a*b+c into FMA, exactly as when the
 * reference itself is built, so the restated loops round like engine.c.
 *
 * ORACLE_LINK_REF: the helper functions come from the reference's
 * inference/core/matvec.c and platform.c (compiled unmodified by
 * oracle/Makefile into oracle/_ref/); otherwise they are restated below.
 * The attention loops live inline in engine.c and are restated in both builds.
 *
 * Parity anchors (tests/test_oracle.py):
 *   - f16 conversion, softmax and rope known answers from tests/test_matvec.c:32-55,
 *     213-239 (copied as numbers into tests/golden/);
 *   - port build == reference build, bit for bit, on every helper and loop.
 */
#include "yattn_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#ifdef ORACLE_LINK_REF
/* --- helpers from the reference (matvec.h / yllm.h declarations) --- */
float    f16_to_f32(uint16_t h);
uint16_t f32_to_f16(float f);
uint64_t yrng(uint64_t* s);
void     softmax(float* v, uint32_t n);
void     rope_inplace(float* v, uint32_t d, uint32_t pos, float theta);
void     rope_inplace_qwen(float* v, uint32_t d, uint32_t pos, float theta);
void     rope_inplace_mrope(float* v, uint32_t head_dim, uint32_t n_dims, uint32_t pos, float theta);
void     l2norm_inplace(float* v, uint32_t n, float eps);
void     gdn_state_update(float* S, float* out, const float* q, const float* k,
                          const float* v, const float* gate, const float* beta,
                          uint32_t num_k_heads, uint32_t hk, uint32_t n_vheads, uint32_t hv);
void     rmsnorm_gated(float* y, const float* x, const uint8_t* w, const float* z,
                       uint32_t n, float eps, uint32_t dtype);
void     rmsnorm(float* y, const float* x, const uint8_t* w, uint32_t n, float eps, uint32_t dtype);
void     conv1d_update(float* state, const float* x, const uint8_t* w, uint32_t dim, uint32_t kwidth);
void     q4k_block(float* y, const uint8_t* blk, uint32_t stride);
void     matmul(float* y, const float* x, const uint8_t* w, uint32_t out, uint32_t in, uint32_t dtype);
#define REF_DT_F16 0u   /* DT_F16, inference/include/llf.h:14 */
#define REF_DT_Q4K 3u   /* DT_Q4K, inference/include/llf.h:17 */
#define REF_DT_F32 1u   /* DT_F32, inference/include/llf.h:15 */

int orc_build_kind(void) { return 1; }
float    orc_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
uint16_t orc_f32_to_f16(float f) { return f32_to_f16(f); }
uint64_t orc_yrng(uint64_t* s) { return yrng(s); }
void orc_softmax(float* v, uint32_t n) { softmax(v, n); }
void orc_rope_inplace(float* v, uint32_t d, uint32_t pos, float theta) { rope_inplace(v, d, pos, theta); }
void orc_rope_inplace_qwen(float* v, uint32_t d, uint32_t pos, float theta) { rope_inplace_qwen(v, d, pos, theta); }
void orc_rope_inplace_mrope(float* v, uint32_t hd, uint32_t n_dims, uint32_t pos, float theta)
{ rope_inplace_mrope(v, hd, n_dims, pos, theta); }
void orc_l2norm_inplace(float* v, uint32_t n, float eps) { l2norm_inplace(v, n, eps); }
void orc_gdn_state_update(float* S, float* out, const float* q, const float* k,
                          const float* v, const float* gate, const float* beta,
                          uint32_t num_k_heads, uint32_t hk, uint32_t n_vheads, uint32_t hv)
{ gdn_state_update(S, out, q, k, v, gate, beta, num_k_heads, hk, n_vheads, hv); }
void orc_rmsnorm_gated_f32(float* y, const float* x, const float* w, const float* z, uint32_t n, float eps)
{ rmsnorm_gated(y, x, (const uint8_t*)w, z, n, eps, REF_DT_F32); }
void orc_rmsnorm(float* y, const float* x, const void* w, uint32_t n, float eps, int w_f16)
{ rmsnorm(y, x, (const uint8_t*)w, n, eps, w_f16 ? REF_DT_F16 : REF_DT_F32); }
void orc_conv1d_update(float* state, float* x, const float* w, uint32_t dim, uint32_t kwidth)
{ conv1d_update(state, x, (const uint8_t*)w, dim, kwidth); }
void orc_q4k_block(float* y, const uint8_t* blk) { q4k_block(y, blk, 0); }
/* the engine's CPU matmul of one token (matvec.c:787-797): fp16 rows, or Q4_K
 * (the AVX2 build quantises x to int8 first, matvec.c:514-520) */
void orc_matmul_f16(float* y, const float* x, const uint16_t* w, uint32_t out, uint32_t in)
{ matmul(y, x, (const uint8_t*)w, out, in, REF_DT_F16); }
void orc_matmul_q4k(float* y, const float* x, const uint8_t* w, uint32_t out, uint32_t in)
{ matmul(y, x, w, out, in, REF_DT_Q4K); }

#else  /* ---------------- restated helpers ("port") ---------------- */

int orc_build_kind(void) { return 0; }

/* platform.c:316-338: exact fp16 -> fp32, subnormals renormalised.  Like the
 * reference, both zeros (0x0000 and 0x8000) come back as +0.0f. */
float orc_f16_to_f32(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t ex = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (ex == 0) {
        if (man == 0) {
            bits = 0;
        } else {
            int shift = 0;
            while ((man & 0x400u) == 0) { man <<= 1; shift++; }
            bits = sign | ((uint32_t)(113 - shift) << 23) | ((man & 0x3ffu) << 13);
        }
    } else if (ex == 0x1f) {
        bits = sign | 0x7f800000u | (man ? 0x7fc000u : 0u);
    } else {
        bits = sign | ((ex + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* platform.c:340-379: fp32 -> fp16 the engine's way: f32 subnormals flush to
 * zero, the normal range rounds half-up on the dropped 13 bits (+0x1000),
 * the fp16-subnormal range rounds half-up at its own shift, overflow -> inf,
 * NaN keeps a quiet payload bit. */
uint16_t orc_f32_to_f16(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t fexp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    int e = (int)fexp - 112;   /* rebias 127 -> 15 */
    if (fexp == 0) return (uint16_t)sign;
    if (fexp == 0xff) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0u));
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        uint32_t full = man | 0x800000u;
        uint32_t sh = (uint32_t)(14 - e);
        return (uint16_t)(sign | ((full + (1u << (sh - 1))) >> sh));
    }
    man += 0x1000u;
    if (man & 0x800000u) {         /* mantissa carried into the exponent */
        e += 1;
        if (e >= 31) return (uint16_t)(sign | 0x7c00u);
        return (uint16_t)(sign | ((uint32_t)e << 10));
    }
    return (uint16_t)(sign | ((uint32_t)e << 10) | (man >> 13));
}

/* platform.c:411-417: splitmix64. */
uint64_t orc_yrng(uint64_t* s)
{
    uint64_t z = (*s += 0x9e3779b97f4a7c15ull);
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

/* matvec.c:1023-1031: max pass, exp+sum pass, divide pass. */
void orc_softmax(float* v, uint32_t n)
{
    float mx = v[0];
    uint32_t i;
    for (i = 1; i < n; i++)
        if (v[i] > mx) mx = v[i];
    float sum = 0.0f;
    for (i = 0; i < n; i++) {
        v[i] = expf(v[i] - mx);
        sum += v[i];
    }
    for (i = 0; i < n; i++) v[i] /= sum;
}

/* matvec.c:890-904: LLaMA pairs (2j, 2j+1). */
void orc_rope_inplace(float* v, uint32_t d, uint32_t pos, float theta)
{
    uint32_t j;
    for (j = 0; j < d / 2; j++) {
        float fr = powf(theta, -2.0f * (float)j / (float)d);
        float ang = fr * (float)pos;
        float c = cosf(ang), s = sinf(ang);
        float a = v[2 * j], b = v[2 * j + 1];
        v[2 * j] = a * c - b * s;
        v[2 * j + 1] = a * s + b * c;
    }
}

/* matvec.c:907-921: qwen2 pairs (j, j + d/2). */
void orc_rope_inplace_qwen(float* v, uint32_t d, uint32_t pos, float theta)
{
    uint32_t half = d / 2, j;
    for (j = 0; j < half; j++) {
        float fr = powf(theta, -2.0f * (float)j / (float)d);
        float ang = fr * (float)pos;
        float c = cosf(ang), s = sinf(ang);
        float a = v[j], b = v[j + half];
        v[j] = a * c - b * s;
        v[j + half] = a * s + b * c;
    }
}

/* matvec.c:924-939: qwen35 M-RoPE on the first n_dims dims, pairs (j, j + n_dims/2). */
void orc_rope_inplace_mrope(float* v, uint32_t hd, uint32_t n_dims, uint32_t pos, float theta)
{
    uint32_t half = n_dims / 2, j;
    (void)hd;
    for (j = 0; j < half; j++) {
        float fr = powf(theta, -2.0f * (float)j / (float)n_dims);
        float ang = fr * (float)pos;
        float c = cosf(ang), s = sinf(ang);
        float a = v[j], b = v[j + half];
        v[j] = a * c - b * s;
        v[j + half] = a * s + b * c;
    }
}

/* matvec.c:942-949: x / max(||x||, eps). */
void orc_l2norm_inplace(float* v, uint32_t n, float eps)
{
    float ss = 0.0f;
    uint32_t i;
    for (i = 0; i < n; i++) ss += v[i] * v[i];
    float scale = 1.0f / fmaxf(sqrtf(ss), eps);
    for (i = 0; i < n; i++) v[i] *= scale;
}

/* matvec.c:975-1004: per v-head h (k-head h % num_k_heads), rows j of the
 * transposed state: decay, delta against k, rank-1 update; then out = S q / sqrt(hv). */
void orc_gdn_state_update(float* S, float* out, const float* q, const float* k,
                          const float* v, const float* gate, const float* beta,
                          uint32_t num_k_heads, uint32_t hk, uint32_t n_vheads, uint32_t hv)
{
    const float scale = 1.0f / sqrtf((float)hv);
    uint32_t h, j, i;
    for (h = 0; h < n_vheads; h++) {
        uint32_t kh = h % num_k_heads;
        const float* qh = q + (size_t)kh * hk;
        const float* kk = k + (size_t)kh * hk;
        const float* vh = v + (size_t)h * hv;
        float* Sh = S + (size_t)h * hk * hv;
        float* oh = out + (size_t)h * hv;
        float g = expf(gate[h]);
        float b = beta[h];
        for (j = 0; j < hv; j++) {
            float* row = Sh + (size_t)j * hv;
            float dot = 0.0f;
            for (i = 0; i < hk; i++) {
                row[i] *= g;
                dot += row[i] * kk[i];
            }
            float del = (vh[j] - dot) * b;
            for (i = 0; i < hk; i++) row[i] += kk[i] * del;
        }
        for (j = 0; j < hv; j++) {
            const float* row = Sh + (size_t)j * hv;
            float dot = 0.0f;
            for (i = 0; i < hk; i++) dot += row[i] * qh[i];
            oh[j] = dot * scale;
        }
    }
}

/* matvec.c:1007-1021 with DT_F32 weights: x * w / sqrt(mean(x^2)+eps) * silu(z). */
void orc_rmsnorm_gated_f32(float* y, const float* x, const float* w, const float* z, uint32_t n, float eps)
{
    float ss = 0.0f;
    uint32_t i;
    for (i = 0; i < n; i++) ss += x[i] * x[i];
    float inv = 1.0f / sqrtf(ss / (float)n + eps);
    for (i = 0; i < n; i++) {
        float zg = z[i];
        y[i] = x[i] * w[i] * inv * (zg / (1.0f + expf(-zg)));
    }
}

/* matvec.c:152-165: y = x * w / sqrt(mean(x^2) + eps), the sum of squares in
 * index order; w is fp32, or fp16 bits (w_f16) widened with f16_to_f32. */
void orc_rmsnorm(float* y, const float* x, const void* w, uint32_t n, float eps, int w_f16)
{
    float s = 0.0f;
    uint32_t i;
    for (i = 0; i < n; i++) s += x[i] * x[i];
    float inv = 1.0f / sqrtf(s / (float)n + eps);
    if (!w_f16) {
        const float* wp = (const float*)w;
        for (i = 0; i < n; i++) y[i] = x[i] * wp[i] * inv;
    } else {
        const uint16_t* wp = (const uint16_t*)w;
        for (i = 0; i < n; i++) y[i] = x[i] * orc_f16_to_f32(wp[i]) * inv;
    }
}

/* matvec.c:956-967: slide x into the newest row of the [kwidth][dim] delay
 * line, then x[ch] = sum over rows i (oldest first) of state[i][ch] * w[ch][i]. */
void orc_conv1d_update(float* state, float* x, const float* w, uint32_t dim, uint32_t kwidth)
{
    uint32_t i, ch;
    memmove(state, state + dim, (size_t)(kwidth - 1) * dim * sizeof(float));
    memcpy(state + (size_t)(kwidth - 1) * dim, x, (size_t)dim * sizeof(float));
    for (ch = 0; ch < dim; ch++) {
        float acc = 0.0f;
        for (i = 0; i < kwidth; i++) acc += state[(size_t)i * dim + ch] * w[(size_t)ch * kwidth + i];
        x[ch] = acc;
    }
}

/* cache.c:174-195: magic (the first 8 bytes of "YLLMSKV01"), n_blocks,
 * kv_dim, max_seq, pos, then for l = 1..n_blocks the first pos rows of K
 * region l and of V region n_blocks + l of the (2*n_blocks + 1)-region blob. */
int orc_sess_kv_save(const uint16_t* kv, uint32_t nb, uint32_t kv_dim, uint32_t max_seq, uint32_t pos,
                     const char* path)
{
    FILE* f = fopen(path, "wb");
    const uint32_t hdr[4] = {nb, kv_dim, max_seq, pos};
    const size_t region = (size_t)max_seq * kv_dim, row = (size_t)pos * kv_dim;
    uint32_t l;
    int rc = 0;
    if (!f) return -1;
    if (fwrite("YLLMSKV0", 1, 8, f) != 8 || fwrite(hdr, 4, 4, f) != 4) rc = -1;
    for (l = 1; !rc && l <= nb; l++) {
        if (fwrite(kv + (size_t)l * region, 2, row, f) != row ||
            fwrite(kv + (size_t)(nb + l) * region, 2, row, f) != row)
            rc = -1;
    }
    fclose(f);
    return rc;
}

/* cache.c:219-247: refuses a file whose magic, n_blocks, kv_dim or max_seq
 * differ from the engine's, or whose pos exceeds max_seq. */
int orc_sess_kv_load(uint16_t* kv, uint32_t nb, uint32_t kv_dim, uint32_t max_seq, const char* path, uint32_t* pos)
{
    FILE* f = fopen(path, "rb");
    char magic[8];
    uint32_t hdr[4];
    uint32_t l;
    int rc = 0;
    if (!f) return -1;
    if (fread(magic, 1, 8, f) != 8 || memcmp(magic, "YLLMSKV0", 8) != 0 || fread(hdr, 4, 4, f) != 4)
        rc = -1;
    else if (hdr[0] != nb || hdr[1] != kv_dim || hdr[2] != max_seq || hdr[3] > max_seq)
        rc = -1;
    else {
        const size_t region = (size_t)max_seq * kv_dim, row = (size_t)hdr[3] * kv_dim;
        for (l = 1; !rc && l <= nb; l++) {
            if (fread(kv + (size_t)l * region, 2, row, f) != row ||
                fread(kv + (size_t)(nb + l) * region, 2, row, f) != row)
                rc = -1;
        }
        if (!rc && pos) *pos = hdr[3];
    }
    fclose(f);
    return rc;
}

/* matvec.c:26-35: 6-bit scale and min of group j from the 12 scale bytes. */
static void scale_min_k4(int j, const uint8_t* q, uint8_t* d, uint8_t* m)
{
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

/* matvec.c:40-59: 256 weights of a 144-byte Q4_K block, d*sc*nib - dmin*mn. */
void orc_q4k_block(float* y, const uint8_t* blk)
{
    float d = orc_f16_to_f32(((const uint16_t*)blk)[0]);
    float mn = orc_f16_to_f32(((const uint16_t*)blk)[1]);
    uint32_t g, e;
    for (g = 0; g < 8; g++) {
        uint8_t sc, m;
        scale_min_k4((int)g, blk + 4, &sc, &m);
        float d1 = d * (float)sc, m1 = mn * (float)m;
        const uint8_t* q = blk + 16 + (g >> 1) * 32;
        for (e = 0; e < 32; e++) {
            uint8_t nib = (g & 1) ? (q[e] >> 4) : (q[e] & 0xF);
            y[g * 32 + e] = d1 * (float)nib - m1;
        }
    }
}

/* matvec.c:111-122 (row-major fp16, fp32 accumulation in index order). */
void orc_matmul_f16(float* y, const float* x, const uint16_t* w, uint32_t out, uint32_t in)
{
    uint32_t oo;
    #pragma omp parallel for schedule(static)
    for (oo = 0; oo < out; oo++) {
        float acc = 0.0f;
        uint32_t ii;
        for (ii = 0; ii < in; ii++) acc += x[ii] * orc_f16_to_f32(w[(size_t)oo * in + ii]);
        y[oo] = acc;
    }
}

void orc_gemv_q4k(float* y, const uint8_t* w, const float* x, uint32_t out, uint32_t in, uint32_t B);
/* The port has no int8 path: its Q4_K matmul is the fp32 one. */
void orc_matmul_q4k(float* y, const float* x, const uint8_t* w, uint32_t out, uint32_t in)
{ orc_gemv_q4k(y, w, x, out, in, 1); }
#endif /* ORACLE_LINK_REF */

int orc_max_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Thread count for the OpenMP loops (launchers such as torchrun export
 * OMP_NUM_THREADS=1; the CPU baseline wants every host core). */
void orc_set_threads(int n)
{
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

void orc_f32_to_f16_buf(const float* src, uint16_t* dst, size_t n)
{
    size_t i;
    for (i = 0; i < n; i++) dst[i] = orc_f32_to_f16(src[i]);
}

void orc_f16_to_f32_buf(const uint16_t* src, float* dst, size_t n)
{
    size_t i;
    for (i = 0; i < n; i++) dst[i] = orc_f16_to_f32(src[i]);
}

/* ---------------- linear layers ---------------- */

/* y[t][o] = sum over the row of x[t][i] * w(o, i) with every Q4_K weight
 * dequantised to fp32 as the reference does (q4k_block, matvec.c:40-59; the
 * same d*sc*nib - dmin*mn as its GPU kernel, cuda_kernels.cu:142-159), summed
 * in index order in fp32.  x [B][in], y [B][out]. */
void orc_gemv_q4k(float* y, const uint8_t* w, const float* x, uint32_t out, uint32_t in, uint32_t B)
{
    const uint32_t nb = in / 256;
    uint32_t t, oo;
    for (t = 0; t < B; t++) {
        #pragma omp parallel for schedule(static)
        for (oo = 0; oo < out; oo++) {
            float tmp[256];
            float acc = 0.0f;
            uint32_t b, e;
            for (b = 0; b < nb; b++) {
                orc_q4k_block(tmp, w + ((size_t)oo * nb + b) * 144);
                for (e = 0; e < 256; e++) acc += x[(size_t)t * in + b * 256 + e] * tmp[e];
            }
            y[(size_t)t * out + oo] = acc;
        }
    }
}

/* The engine's fp16 matmul (matvec.c:111-122) for each of B tokens. */
void orc_gemv_f16(float* y, const uint16_t* w, const float* x, uint32_t out, uint32_t in, uint32_t B)
{
    uint32_t t;
    for (t = 0; t < B; t++) orc_matmul_f16(y + (size_t)t * out, x + (size_t)t * in, w, out, in);
}

/* ---------------- qwen35 GDN layer inputs ---------------- */

/* engine.c:785-821 for T tokens of each of n_seqs sequences, token by token:
 * gates (beta = sigmoid, gate = softplus(alpha + dt) * A), conv1d_update of
 * the projection into the delay line, silu, then the q / k / v split with
 * l2norm_inplace of every q and k head.  Layouts: qkv [n_seqs][T][conv_chan],
 * conv_state [n_seqs][kwidth][conv_chan], conv_w [conv_chan][kwidth], alpha /
 * beta_in / gate / beta [n_seqs][T][nv], q / k [n_seqs][T][nk*hk], v
 * [n_seqs][T][nv*hv].  qkv is not modified. */
void orc_gdn_inputs(const float* qkv, float* conv_state, const float* conv_w, const float* alpha,
                    const float* beta_in, const float* dt, const float* a, float* q, float* k, float* v,
                    float* gate, float* beta, uint32_t n_seqs, uint32_t T, uint32_t conv_chan, uint32_t kwidth,
                    uint32_t nk, uint32_t hk, uint32_t nv, uint32_t hv, float eps)
{
    const uint32_t key_dim = nk * hk, value_dim = nv * hv;
    float* x = (float*)malloc((size_t)conv_chan * sizeof(float));
    uint32_t s, t, h, ch;
    if (!x) return;
    for (s = 0; s < n_seqs; s++) {
        float* st = conv_state + (size_t)s * kwidth * conv_chan;
        for (t = 0; t < T; t++) {
            const size_t row = (size_t)s * T + t;
            for (h = 0; h < nv; h++) {
                const size_t i = row * nv + h;
                beta[i] = 1.0f / (1.0f + expf(-beta_in[i]));
                float ab = alpha[i] + dt[h];
                float sp = log1pf(expf(ab));
                gate[i] = sp * a[h];
            }
            memcpy(x, qkv + row * conv_chan, (size_t)conv_chan * sizeof(float));
            orc_conv1d_update(st, x, conv_w, conv_chan, kwidth);
            for (ch = 0; ch < conv_chan; ch++) x[ch] = x[ch] / (1.0f + expf(-x[ch]));
            for (h = 0; h < nk; h++) orc_l2norm_inplace(x + (size_t)h * hk, hk, eps);
            for (h = 0; h < nk; h++) orc_l2norm_inplace(x + key_dim + (size_t)h * hk, hk, eps);
            memcpy(q + row * key_dim, x, (size_t)key_dim * sizeof(float));
            memcpy(k + row * key_dim, x + key_dim, (size_t)key_dim * sizeof(float));
            memcpy(v + row * value_dim, x + 2 * key_dim, (size_t)value_dim * sizeof(float));
        }
    }
    free(x);
}

/* ---------------- one token's RoPE + KV store ---------------- */

/* engine.c:1052-1072 (llama / qwen pairs over the whole head) and
 * engine.c:921-934 (qwen35 M-RoPE over the first n_dims dims): every q head
 * and k head rotated in place at pos, then k and v rounded into cache row pos.
 * kind 0 llama, 1 qwen, 2 mrope. */
void orc_rope_store(float* q, float* k, const float* v, uint16_t* kcache, uint16_t* vcache,
                    uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t kv_dim, int kind,
                    uint32_t n_dims, uint32_t pos, float theta)
{
    uint32_t hh, j;
    for (hh = 0; hh < n_heads + n_kv; hh++) {
        float* x = hh < n_heads ? q + (size_t)hh * hd : k + (size_t)(hh - n_heads) * hd;
        if (kind == 0)
            orc_rope_inplace(x, hd, pos, theta);
        else if (kind == 1)
            orc_rope_inplace_qwen(x, hd, pos, theta);
        else
            orc_rope_inplace_mrope(x, hd, n_dims, pos, theta);
    }
    for (j = 0; j < kv_dim; j++) {
        kcache[(size_t)pos * kv_dim + j] = orc_f32_to_f16(k[j]);
        vcache[(size_t)pos * kv_dim + j] = orc_f32_to_f16(v[j]);
    }
}

/* QK-norm before the rotation: engine.c:915-919 (qwen35, then M-RoPE 922-925)
 * and 1036-1045 (qwen3): rmsnorm of every q head and every k head with the
 * layer's shared head_dim weights, then orc_rope_store. */
void orc_qknorm_rope_store(float* q, float* k, const float* v, uint16_t* kcache, uint16_t* vcache,
                           uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t kv_dim, int kind,
                           uint32_t n_dims, uint32_t pos, float theta, const void* q_w, const void* k_w,
                           int w_f16, float eps)
{
    uint32_t hh;
    for (hh = 0; hh < n_heads; hh++) orc_rmsnorm(q + (size_t)hh * hd, q + (size_t)hh * hd, q_w, hd, eps, w_f16);
    for (hh = 0; hh < n_kv; hh++) orc_rmsnorm(k + (size_t)hh * hd, k + (size_t)hh * hd, k_w, hd, eps, w_f16);
    orc_rope_store(q, k, v, kcache, vcache, n_heads, n_kv, hd, kv_dim, kind, n_dims, pos, theta);
}

/* ---------------- attention loops (engine.c, operation order kept) ---------------- */

/* One head of the engine's decode/prefill inner body: scores over keys
 * 0..pos (acc over head_dim, then * inv_d), softmax, then the PV sum.
 * engine.c:1078-1095 and 541-561 are the same body. */
static void head_attend(float* out, const float* qh, const uint16_t* kcache, const uint16_t* vcache,
                        uint32_t pos, uint32_t kv_head, uint32_t hd, uint32_t kv_dim, float* att_h)
{
    float inv_d = 1.0f / sqrtf((float)hd);
    uint32_t s, jj;
    for (s = 0; s <= pos; s++) {
        const uint16_t* kh = kcache + (size_t)s * kv_dim + (size_t)kv_head * hd;
        float acc = 0.0f;
        for (jj = 0; jj < hd; jj++) acc += qh[jj] * orc_f16_to_f32(kh[jj]);
        att_h[s] = acc * inv_d;
    }
    orc_softmax(att_h, pos + 1);
    memset(out, 0, (size_t)hd * 4);
    for (s = 0; s <= pos; s++) {
        const uint16_t* vh = vcache + (size_t)s * kv_dim + (size_t)kv_head * hd;
        float a = att_h[s];
        for (jj = 0; jj < hd; jj++) out[jj] += a * orc_f16_to_f32(vh[jj]);
    }
}

void orc_attn_decode(float* att_out, const float* q, const uint16_t* kcache, const uint16_t* vcache,
                     uint32_t pos, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                     uint32_t kv_dim)
{
    float* att = (float*)malloc((size_t)n_heads * (pos + 1) * sizeof(float));
    int hh;
    #pragma omp parallel for schedule(static)
    for (hh = 0; hh < (int)n_heads; hh++) {
        uint32_t kv_head = (uint32_t)hh * n_kv_heads / n_heads;
        head_attend(att_out + (size_t)hh * head_dim, q + (size_t)hh * head_dim, kcache, vcache,
                    pos, kv_head, head_dim, kv_dim, att + (size_t)hh * (pos + 1));
    }
    free(att);
}

void orc_attn_prefill(float* att_out, const float* q, const uint16_t* kcache, const uint16_t* vcache,
                      uint32_t pos_start, uint32_t B, uint32_t n_heads, uint32_t n_kv_heads,
                      uint32_t head_dim, uint32_t kv_dim, uint32_t q_stride)
{
    uint32_t maxlen = pos_start + B;
    int nth = orc_max_threads();
    float* att = (float*)malloc((size_t)nth * maxlen * sizeof(float));
    int hh;
    #pragma omp parallel for schedule(static)
    for (hh = 0; hh < (int)n_heads; hh++) {
        int tid = 0;
#ifdef _OPENMP
        tid = omp_get_thread_num();
#endif
        uint32_t kv_head = (uint32_t)hh * n_kv_heads / n_heads;
        uint32_t bb;
        for (bb = 0; bb < B; bb++) {
            head_attend(att_out + (size_t)bb * q_stride + (size_t)hh * head_dim,
                        q + (size_t)bb * q_stride + (size_t)hh * head_dim, kcache, vcache,
                        pos_start + bb, kv_head, head_dim, kv_dim, att + (size_t)tid * maxlen);
        }
    }
    free(att);
}

/* engine.c:958-960: the gate pass runs after every head's attention. */
static void sigmoid_gate(float* att_out, const float* gate, size_t n)
{
    size_t i;
    for (i = 0; i < n; i++) att_out[i] *= 1.0f / (1.0f + expf(-gate[i]));
}

void orc_attn_decode_gated(float* att_out, const float* q, const float* gate,
                           const uint16_t* kcache, const uint16_t* vcache,
                           uint32_t pos, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                           uint32_t kv_dim)
{
    orc_attn_decode(att_out, q, kcache, vcache, pos, n_heads, n_kv_heads, head_dim, kv_dim);
    sigmoid_gate(att_out, gate, (size_t)n_heads * head_dim);
}

void orc_attn_prefill_gated(float* att_out, const float* q, const float* gate,
                            const uint16_t* kcache, const uint16_t* vcache,
                            uint32_t pos_start, uint32_t B, uint32_t n_heads, uint32_t n_kv_heads,
                            uint32_t head_dim, uint32_t kv_dim, uint32_t q_stride)
{
    uint32_t bb;
    orc_attn_prefill(att_out, q, kcache, vcache, pos_start, B, n_heads, n_kv_heads, head_dim,
                     kv_dim, q_stride);
    for (bb = 0; bb < B; bb++)
        sigmoid_gate(att_out + (size_t)bb * q_stride, gate + (size_t)bb * q_stride,
                     (size_t)n_heads * head_dim);
}

void orc_gdn_step(float* S, float* out, const float* q, const float* k, const float* v,
                  const float* gate, const float* beta, uint32_t num_k_heads, uint32_t hk,
                  uint32_t n_vheads, uint32_t hv, const float* norm_w, const float* z, float eps)
{
    int h;
    /* One reference call per head (num_k_heads = n_vheads = 1 on offset
     * pointers) does exactly the arithmetic of the all-heads call. */
    #pragma omp parallel for schedule(static)
    for (h = 0; h < (int)n_vheads; h++) {
        uint32_t kh = (uint32_t)h % num_k_heads;
        orc_gdn_state_update(S + (size_t)h * hk * hv, out + (size_t)h * hv, q + (size_t)kh * hk,
                             k + (size_t)kh * hk, v + (size_t)h * hv, gate + h, beta + h, 1, hk, 1, hv);
        if (norm_w && z)
            orc_rmsnorm_gated_f32(out + (size_t)h * hv, out + (size_t)h * hv, norm_w,
                                  z + (size_t)h * hv, hv, eps);
    }
}

void orc_gdn_prefill(float* S, float* out, const float* q, const float* k, const float* v,
                     const float* gate, const float* beta, uint32_t T, uint32_t num_k_heads,
                     uint32_t hk, uint32_t n_vheads, uint32_t hv,
                     const float* norm_w, const float* z, float eps)
{
    int h;
    size_t qk_row = (size_t)num_k_heads * hk, v_row = (size_t)n_vheads * hv;
    #pragma omp parallel for schedule(dynamic, 1)
    for (h = 0; h < (int)n_vheads; h++) {
        uint32_t kh = (uint32_t)h % num_k_heads;
        uint32_t t;
        for (t = 0; t < T; t++) {
            float* oh = out + t * v_row + (size_t)h * hv;
            orc_gdn_state_update(S + (size_t)h * hk * hv, oh, q + t * qk_row + (size_t)kh * hk,
                                 k + t * qk_row + (size_t)kh * hk, v + t * v_row + (size_t)h * hv,
                                 gate + (size_t)t * n_vheads + h, beta + (size_t)t * n_vheads + h,
                                 1, hk, 1, hv);
            if (norm_w && z)
                orc_rmsnorm_gated_f32(oh, oh, norm_w, z + t * v_row + (size_t)h * hv, hv, eps);
        }
    }
}

/* ---------------- deterministic seeded inputs ----------------
 * The GPU generator in yllm_b200/csrc/fixture.cu performs this exact sequence
 * of IEEE operations.  Literals are the nearest doubles of the named values. */

#define D_SQRT2    1.4142135623730951      /* sqrt(2) */
#define D_LN2      0.6931471805599453      /* ln 2 */
#define D_LN2_HI   0.6931471803691238      /* ln 2 to 32 bits */
#define D_LN2_LO   1.9082149292705877e-10  /* ln 2 - D_LN2_HI */
#define D_INV_LN2  1.4426950408889634
#define D_2_PI     0.6366197723675814      /* 2/pi */
#define D_PIO2_1   1.5707963267341256      /* pi/2 to 33 bits */
#define D_PIO2_2   6.077100506303966e-11   /* next 33 bits */
#define D_PIO2_3   2.0222662487959506e-21  /* remainder */
#define D_2PI      6.283185307179586

/* ln x = e ln2 + 2 atanh((m-1)/(m+1)), m in [sqrt(2)/2, sqrt(2)];
 * atanh series s + s^3/3 + ... + s^23/23 (|s| <= 0.1716). */
double orc_det_log(double x)
{
    uint64_t b;
    memcpy(&b, &x, 8);
    int e = (int)((b >> 52) & 0x7ff) - 1023;
    b = (b & 0x000fffffffffffffull) | 0x3ff0000000000000ull;
    double m;
    memcpy(&m, &b, 8);
    if (m > D_SQRT2) { m = m * 0.5; e += 1; }
    double s = (m - 1.0) / (m + 1.0);
    double s2 = s * s;
    double p = 0.043478260869565216;           /* 1/23 */
    p = fma(p, s2, 0.047619047619047616);      /* 1/21 */
    p = fma(p, s2, 0.05263157894736842);       /* 1/19 */
    p = fma(p, s2, 0.058823529411764705);      /* 1/17 */
    p = fma(p, s2, 0.06666666666666667);       /* 1/15 */
    p = fma(p, s2, 0.07692307692307693);       /* 1/13 */
    p = fma(p, s2, 0.09090909090909091);       /* 1/11 */
    p = fma(p, s2, 0.1111111111111111);        /* 1/9 */
    p = fma(p, s2, 0.14285714285714285);       /* 1/7 */
    p = fma(p, s2, 0.2);                       /* 1/5 */
    p = fma(p, s2, 0.3333333333333333);        /* 1/3 */
    double t = (s * s2) * p;
    double lm = fma(2.0, t, 2.0 * s);
    return fma((double)e, D_LN2, lm);
}

/* e^x = 2^k e^r, k = rint(x/ln2), r by a two-part ln2; Taylor series to r^13. */
double orc_det_exp(double x)
{
    double k = rint(x * D_INV_LN2);
    double r = fma(-k, D_LN2_HI, x);
    r = fma(-k, D_LN2_LO, r);
    double p = 1.6059043836821613e-10;         /* 1/13! */
    p = fma(p, r, 2.08767569878681e-09);       /* 1/12! */
    p = fma(p, r, 2.505210838544172e-08);      /* 1/11! */
    p = fma(p, r, 2.755731922398589e-07);      /* 1/10! */
    p = fma(p, r, 2.7557319223985893e-06);     /* 1/9! */
    p = fma(p, r, 2.48015873015873e-05);       /* 1/8! */
    p = fma(p, r, 0.0001984126984126984);      /* 1/7! */
    p = fma(p, r, 0.001388888888888889);       /* 1/6! */
    p = fma(p, r, 0.008333333333333333);       /* 1/5! */
    p = fma(p, r, 0.041666666666666664);       /* 1/4! */
    p = fma(p, r, 0.16666666666666666);        /* 1/3! */
    p = fma(p, r, 0.5);
    p = fma(p, r, 1.0);
    p = fma(p, r, 1.0);
    int64_t ki = (int64_t)k;
    uint64_t sb = (uint64_t)(ki + 1023) << 52;
    double sc;
    memcpy(&sc, &sb, 8);
    return p * sc;
}

/* Cody-Waite reduction by pi/2 (three parts), then Taylor series on |r| <= pi/4:
 * sin to r^17, cos to r^18. */
void orc_det_sincos(double x, double* s_out, double* c_out)
{
    double k = rint(x * D_2_PI);
    double r = fma(-k, D_PIO2_1, x);
    r = fma(-k, D_PIO2_2, r);
    r = fma(-k, D_PIO2_3, r);
    double r2 = r * r;
    double ps = 2.8114572543455206e-15;        /* 1/17! */
    ps = fma(ps, r2, -7.647163731819816e-13);  /* -1/15! */
    ps = fma(ps, r2, 1.6059043836821613e-10);  /* 1/13! */
    ps = fma(ps, r2, -2.505210838544172e-08);  /* -1/11! */
    ps = fma(ps, r2, 2.7557319223985893e-06);  /* 1/9! */
    ps = fma(ps, r2, -0.0001984126984126984);  /* -1/7! */
    ps = fma(ps, r2, 0.008333333333333333);    /* 1/5! */
    ps = fma(ps, r2, -0.16666666666666666);    /* -1/3! */
    double sn = fma(r * r2, ps, r);
    double pc = -1.5619206968586225e-16;       /* -1/18! */
    pc = fma(pc, r2, 4.779477332387385e-14);   /* 1/16! */
    pc = fma(pc, r2, -1.1470745597729725e-11); /* -1/14! */
    pc = fma(pc, r2, 2.08767569878681e-09);    /* 1/12! */
    pc = fma(pc, r2, -2.755731922398589e-07);  /* -1/10! */
    pc = fma(pc, r2, 2.48015873015873e-05);    /* 1/8! */
    pc = fma(pc, r2, -0.001388888888888889);   /* -1/6! */
    pc = fma(pc, r2, 0.041666666666666664);    /* 1/4! */
    pc = fma(pc, r2, -0.5);
    double cs = fma(pc, r2, 1.0);
    int64_t q = ((int64_t)k) & 3;
    if (q == 0)      { *s_out = sn;  *c_out = cs;  }
    else if (q == 1) { *s_out = cs;  *c_out = -sn; }
    else if (q == 2) { *s_out = -sn; *c_out = -cs; }
    else             { *s_out = -cs; *c_out = sn;  }
}

/* The k-th (0-based) yrng() output of a stream whose state starts at `seed`
 * (ysrand maps 0 to the golden-ratio constant, platform.c:405-409). */
uint64_t orc_stream_draw(uint64_t seed, uint64_t k)
{
    if (seed == 0) seed = 0x9e3779b97f4a7c15ull;
    uint64_t st = seed + k * 0x9e3779b97f4a7c15ull;
    return orc_yrng(&st);
}

/* Box-Muller on draw i/2: u1 = (top 24 bits + 1) / 2^24 in (0,1] (the engine's
 * uniform, engine.c:1649, shifted off zero), u2 = next 24 bits / 2^24;
 * even i -> r cos(2 pi u2), odd i -> r sin(2 pi u2). */
double orc_normal_d(uint64_t seed, uint64_t i)
{
    uint64_t v = orc_stream_draw(seed, i >> 1);
    double u1 = (double)((v >> 40) + 1) * 5.9604644775390625e-08;       /* 2^-24 */
    double u2 = (double)((v >> 16) & 0xffffffull) * 5.9604644775390625e-08;
    double r = sqrt(-2.0 * orc_det_log(u1));
    double sn, cs;
    orc_det_sincos(D_2PI * u2, &sn, &cs);
    return (i & 1) ? r * sn : r * cs;
}

void orc_fill_normal(uint64_t seed, uint64_t first, size_t n, double scale, float* out)
{
    long long i;
    #pragma omp parallel for schedule(static)
    for (i = 0; i < (long long)n; i++)
        out[i] = (float)(orc_normal_d(seed, first + (uint64_t)i) * scale);
}

void orc_rope_rows(float* x, size_t n_rows, uint32_t n_heads, uint32_t hd, uint32_t pos0, double theta)
{
    double lt = orc_det_log(theta);
    uint32_t half = hd / 2;
    long long r;
    #pragma omp parallel for schedule(static)
    for (r = 0; r < (long long)n_rows; r++) {
        double pos = (double)(pos0 + (uint32_t)r);
        uint32_t h, j;
        for (j = 0; j < half; j++) {
            double t = (double)(2 * j) / (double)hd;
            double fr = orc_det_exp(-(t * lt));
            double sn, cs;
            orc_det_sincos(pos * fr, &sn, &cs);
            for (h = 0; h < n_heads; h++) {
                float* v = x + (size_t)r * n_heads * hd + (size_t)h * hd;
                double a = (double)v[j], b = (double)v[j + half];
                v[j] = (float)fma(a, cs, -(b * sn));
                v[j + half] = (float)fma(a, sn, b * cs);
            }
        }
    }
}

void orc_round_f16(const float* x, size_t n, uint16_t* out)
{
    long long i;
    #pragma omp parallel for schedule(static)
    for (i = 0; i < (long long)n; i++) out[i] = orc_f32_to_f16(x[i]);
}

void orc_round_f16_inplace(float* x, size_t n)
{
    long long i;
    #pragma omp parallel for schedule(static)
    for (i = 0; i < (long long)n; i++) x[i] = orc_f16_to_f32(orc_f32_to_f16(x[i]));
}

void orc_round_bf16_inplace(float* x, size_t n)
{
    size_t i;
    for (i = 0; i < n; i++) {
        uint32_t b;
        memcpy(&b, &x[i], 4);
        b &= 0xffff0000u;
        memcpy(&x[i], &b, 4);
    }
}

/* gate = -softplus(z_a) = -ln(1 + e^z_a), so e^gate is the decay alpha;
 * beta = 1 / (1 + e^-z_b). */
void orc_gdn_gates(uint64_t seed_a, uint64_t seed_b, uint64_t first, size_t n, float* gate, float* beta)
{
    size_t i;
    for (i = 0; i < n; i++) {
        double za = orc_normal_d(seed_a, first + i);
        double zb = orc_normal_d(seed_b, first + i);
        gate[i] = (float)(-orc_det_log(1.0 + orc_det_exp(za)));
        beta[i] = (float)(1.0 / (1.0 + orc_det_exp(-zb)));
    }
}

void orc_gdn_qk(uint64_t seed, uint64_t first_row, size_t n_rows, uint32_t n_heads, uint32_t hd,
                float eps, float* out)
{
    size_t row = (size_t)n_heads * hd;
    orc_fill_normal(seed, first_row * row, n_rows * row, 1.0, out);
    orc_round_bf16_inplace(out, n_rows * row);
    size_t i;
    for (i = 0; i < n_rows * n_heads; i++) orc_l2norm_inplace(out + i * hd, hd, eps);
}

uint32_t orc_ctx_len(uint64_t seed, uint32_t i, uint32_t lo, uint32_t hi)
{
    uint64_t v = orc_stream_draw(seed, i);
    return lo + (uint32_t)(v % (uint64_t)(hi - lo + 1));
}

uint64_t orc_fnv1a(const void* p, size_t n)
{
    const unsigned char* c = (const unsigned char*)p;
    uint64_t h = 0xcbf29ce484222325ull;
    size_t i;
    for (i = 0; i < n; i++) { h ^= c[i]; h *= 0x100000001b3ull; }
    return h;
}

uint64_t orc_checksum64(const void* p, size_t n)
{
    const uint64_t* w = (const uint64_t*)p;
    size_t n_words = n / 8, per = 65536 / 8;
    size_t n_blocks = (n + 65535) / 65536;
    uint64_t* hb = (uint64_t*)malloc((n_blocks ? n_blocks : 1) * sizeof(uint64_t));
    long long b;
    #pragma omp parallel for schedule(static)
    for (b = 0; b < (long long)n_blocks; b++) {
        size_t i0 = (size_t)b * per, i1 = i0 + per < n_words ? i0 + per : n_words, i;
        uint64_t h = 0xcbf29ce484222325ull;
        for (i = i0; i < i1; i++) { h ^= w[i]; h *= 0x100000001b3ull; }
        hb[b] = h;
    }
    uint64_t h = 0xcbf29ce484222325ull;
    size_t j;
    for (j = 0; j < n_blocks; j++) { h ^= hb[j]; h *= 0x100000001b3ull; }
    free(hb);
    return h;
}
