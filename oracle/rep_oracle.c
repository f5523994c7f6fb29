/*
 * rep_oracle.c -- CPU restatement of the RepEncoder W8A8 hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA path is
 * compared against; it is never linked into, loaded by, or called from the
 * product library.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it.
 *
 * Every function restates one piece of the reference (YuDeng0102/baidu_cti_grab)
 * in plain C with the floating-point operations spelled out one IEEE op at a
 * time (no contraction: build with -ffp-contract=off), so that the CUDA
 * kernels, which issue the same ops with explicit __f*_rn intrinsics, can be
 * checked bit for bit:
 *
 *   rbo_embedding_bag_sum   models.py:17,27-33   nn.EmbeddingBag(mode='sum',
 *                           padding_idx=0) after values.clamp(0, V-1); fp32
 *                           accumulation in bag order, one RNE round to the
 *                           table dtype.  The last bag runs to the end of
 *                           `values` (offsets[:-1] is what the reference passes).
 *   rbo_layernorm_row       models.py:21,45 nn.LayerNorm(S*D, eps) over the
 *                           concatenated row, restated as a two-pass fp32
 *                           LayerNorm whose reduction order is fixed (the
 *                           "canonical order" below) so it is reproducible.
 *   rbo_quant_dynamic_v2    quantization/w8a8_triton_kernels.py:41-64
 *   rbo_quant_static_v2     quantization/w8a8_triton_kernels.py:23-38
 *   rbo_quant_rows_v1       kernels/quantization.py:6-35
 *   rbo_gemm_i8_i32         quantization/w8a8_triton_kernels.py:67-171 (int32 acc)
 *   rbo_scaled_epilogue     quantization/w8a8_triton_kernels.py:230-246
 *   rbo_rep_forward         models.py:24-48 + w8a8_linear's quantiser, i.e.
 *                           gather -> pool -> concat -> LN -> int8 quant.
 *
 * Canonical LayerNorm reduction order (shared with the CUDA kernel): a row of
 * S slots x 512 columns is reduced slot by slot.  Inside a slot, "lane" l
 * (0..31) owns 16 elements, columns 8l..8l+7 then 256+8l..256+8l+7; walking
 * them in that order, elements at even positions accumulate into a0 and odd
 * positions into a1 (both from 0.0f), and the lane partial is a0 + a1; the
 * 32 lane partials are combined by an xor-butterfly with distances 16, 8, 4,
 * 2, 1 (p[l] = p[l] + p[l^d]).  (The even/odd split is what a packed two-wide
 * fp32 add computes.)  Per slot s this order gives the sum T_s of x and, with
 * the slot mean m_s = T_s / 512, the centred square sum Q_s of (x - m_s)^2
 * (fmaf(d, d, acc) per element).  The slots are then combined by the same
 * 32-wide xor-butterfly, slot s in position s and 0.0f in positions S..31:
 *   mean = butterfly_s(T_s) / H
 *   M2   = butterfly_s(Q_s + 512 * (m_s - mean)^2)   (Chan's parallel update)
 *   var  = M2 / H;  rstd = 1.0f / sqrtf(var + eps)
 *   y    = fmaf(rstd * (x - mean), gamma, beta)   (then RNE to the row dtype)
 * Division and square root are IEEE correctly rounded here and in the kernel.
 */
#include <stdint.h>
#include <string.h>
#include <math.h>
#include <stdlib.h>
#include <pthread.h>

enum { RBO_F32 = 0, RBO_BF16 = 1, RBO_F16 = 2, RBO_I32 = 3 };

/* ----------------------------------------------------------------- dtypes */
static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u);                                            /* RNE */
    return (uint16_t)(u >> 16);
}

static inline float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu, u;
    if (exp == 0) {
        if (man == 0) {
            u = sign;
        } else { /* subnormal */
            float f = ldexpf((float)man, -24);
            memcpy(&u, &f, 4);
            u |= sign;
        }
    } else if (exp == 31) {
        u = sign | 0x7f800000u | (man << 13);
    } else {
        u = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint16_t f32_to_f16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    float a = fabsf(f);
    if (a != a) return sign | 0x7e00u;
    if (a >= 65520.0f) return sign | 0x7c00u; /* rounds to inf */
    if (a < 6.103515625e-05f) {               /* subnormal range: quantum 2^-24 */
        float q = a * 16777216.0f;             /* exact scaling by 2^24 */
        float r = nearbyintf(q);               /* RNE under default rounding mode */
        return sign | (uint16_t)r;
    }
    uint32_t au;
    memcpy(&au, &a, 4);
    uint32_t exp = (au >> 23) - 112u;
    uint32_t man = au & 0x7fffffu;
    uint32_t half = (exp << 10) | (man >> 13);
    uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (half & 1u))) half += 1u;
    return sign | (uint16_t)half;
}

static inline float load_elem(const void* p, int dtype, int64_t i) {
    switch (dtype) {
        case RBO_BF16: return bf16_to_f32(((const uint16_t*)p)[i]);
        case RBO_F16: return f16_to_f32(((const uint16_t*)p)[i]);
        default: return ((const float*)p)[i];
    }
}

static inline void store_elem(void* p, int dtype, int64_t i, float v) {
    switch (dtype) {
        case RBO_BF16: ((uint16_t*)p)[i] = f32_to_bf16(v); break;
        case RBO_F16: ((uint16_t*)p)[i] = f32_to_f16(v); break;
        default: ((float*)p)[i] = v; break;
    }
}

/* round a value to `dtype` and back (identity for fp32) */
static inline float round_to(int dtype, float v) {
    switch (dtype) {
        case RBO_BF16: return bf16_to_f32(f32_to_bf16(v));
        case RBO_F16: return f16_to_f32(f32_to_f16(v));
        default: return v;
    }
}

void rbo_round_to_dtype(const float* x, int64_t n, int dtype, void* out) {
    for (int64_t i = 0; i < n; ++i) store_elem(out, dtype, i, x[i]);
}

void rbo_dtype_to_f32(const void* x, int64_t n, int dtype, float* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = load_elem(x, dtype, i);
}

/* ------------------------------------------------------- embedding bag sum */
/*
 * models.py:27-33: values.clamp(0, V-1), then EmbeddingBag(sum, padding_idx=0)
 * with offsets[:-1].  Bag i covers values[offsets[i] : offsets[i+1]] for
 * i < N-1 and values[offsets[N-1] : nnz] for the last bag.  Ends are clamped
 * to [start, nnz]; an empty bag pools to 0.  out is [N, D] in out_dtype.
 */
void rbo_embedding_bag_sum(const void* table, int table_dtype, int64_t num_rows, int64_t dim,
                           const int64_t* values, int64_t nnz, const int64_t* offsets,
                           int64_t n_items, void* out, int out_dtype) {
    float* acc = (float*)malloc(sizeof(float) * (size_t)dim);
    for (int64_t i = 0; i < n_items; ++i) {
        int64_t start = offsets[i];
        int64_t end = (i + 1 < n_items) ? offsets[i + 1] : nnz;
        if (start < 0) start = 0;
        if (start > nnz) start = nnz;
        if (end > nnz) end = nnz;
        for (int64_t d = 0; d < dim; ++d) acc[d] = 0.0f;
        for (int64_t j = start; j < end; ++j) {
            int64_t id = values[j];
            if (id < 0) id = 0;
            if (id > num_rows - 1) id = num_rows - 1;
            if (id == 0) continue; /* padding_idx rows are excluded */
            for (int64_t d = 0; d < dim; ++d) acc[d] = acc[d] + load_elem(table, table_dtype, id * dim + d);
        }
        for (int64_t d = 0; d < dim; ++d) store_elem(out, out_dtype, i * dim + d, acc[d]);
    }
    free(acc);
}

/* --------------------------------------------------- canonical LayerNorm */
/* p[0] after the xor-butterfly p[l] = p[l] + p[l^d], d = 16, 8, 4, 2, 1 */
static float butterfly32(float* p) {
    for (int dist = 16; dist >= 1; dist >>= 1) {
        float q[32];
        for (int l = 0; l < 32; ++l) q[l] = p[l] + p[l ^ dist];
        memcpy(p, q, 32 * sizeof(float));
    }
    return p[0];
}

static float canonical_slot_sum(const float* seg, float mean, int centred) {
    float p[32];
    for (int l = 0; l < 32; ++l) {
        /* lane l's 16 columns in order; even positions feed a0, odd positions a1 */
        float a[2] = {0.0f, 0.0f};
        for (int e = 0; e < 16; ++e) {
            const int col = (e < 8) ? 8 * l + e : 256 + 8 * l + (e - 8);
            float v = seg[col];
            if (centred) {
                float d = v - mean;
                a[e & 1] = fmaf(d, d, a[e & 1]);
            } else {
                a[e & 1] = a[e & 1] + v;
            }
        }
        p[l] = a[0] + a[1];
    }
    return butterfly32(p);
}

/*
 * LayerNorm of one row x[S*512] (values already in the row dtype, widened to
 * fp32).  gamma/beta widened to fp32.  y receives fp32 values rounded to
 * out_dtype (so y[] holds exactly what the kernel stores).  mean/rstd out.
 * 1 <= n_slots <= 32 (the slots are combined by a 32-wide butterfly).
 */
void rbo_layernorm_row(const float* x, int64_t n_slots, const float* gamma, const float* beta,
                       float eps, int out_dtype, float* y, float* mean_out, float* rstd_out) {
    const int64_t H = n_slots * 512;
    float slot_sum[32], slot_q[32], p[32];
    for (int64_t s = 0; s < 32; ++s) {
        slot_sum[s] = 0.0f;
        slot_q[s] = 0.0f;
    }
    for (int64_t s = 0; s < n_slots; ++s) {
        slot_sum[s] = canonical_slot_sum(x + s * 512, 0.0f, 0);
        const float m_s = slot_sum[s] / 512.0f;
        slot_q[s] = canonical_slot_sum(x + s * 512, m_s, 1);
    }
    memcpy(p, slot_sum, sizeof(p));
    const float mean = butterfly32(p) / (float)H;
    /* Chan's combination of the per-slot centred sums, butterfly over slots */
    for (int64_t s = 0; s < 32; ++s) {
        const float d = slot_sum[s] / 512.0f - mean;
        p[s] = s < n_slots ? slot_q[s] + 512.0f * (d * d) : 0.0f;
    }
    const float var = butterfly32(p) / (float)H;
    const float rstd = 1.0f / sqrtf(var + eps);
    for (int64_t k = 0; k < H; ++k) {
        float d = x[k] - mean;
        float t = rstd * d;
        y[k] = round_to(out_dtype, fmaf(t, gamma[k], beta[k]));
    }
    if (mean_out) *mean_out = mean;
    if (rstd_out) *rstd_out = rstd;
}

/* ------------------------------------------------------------ quantisers */
static inline int8_t clamp_i8(float q, float lo, float hi) {
    if (q < lo) q = lo;
    if (q > hi) q = hi;
    return (int8_t)q;
}

/* w8a8_triton_kernels.py:56-64: amax = max(max|x|, 1e-8); scale = amax/127;
 * q = clamp(round_half_away(x * (127/amax)), -128, 127). */
void rbo_quant_dynamic_v2(const float* x, int64_t rows, int64_t cols, int8_t* q, float* scale) {
    for (int64_t r = 0; r < rows; ++r) {
        const float* xr = x + r * cols;
        float amax = 0.0f;
        for (int64_t k = 0; k < cols; ++k) amax = fmaxf(amax, fabsf(xr[k]));
        amax = fmaxf(amax, 1e-8f);
        float s = amax / 127.0f;
        float inv = 127.0f / amax;
        for (int64_t k = 0; k < cols; ++k) q[r * cols + k] = clamp_i8(roundf(xr[k] * inv), -128.0f, 127.0f);
        scale[r] = s;
    }
}

/* w8a8_triton_kernels.py:34-37: q = clamp(round_half_away(x * (1/s)), -128, 127). */
void rbo_quant_static_v2(const float* x, int64_t n, float s, int8_t* q) {
    float inv = 1.0f / s;
    for (int64_t i = 0; i < n; ++i) q[i] = clamp_i8(roundf(x[i] * inv), -128.0f, 127.0f);
}

/* kernels/quantization.py:24-35: scale = max(amax/127, 1e-8);
 * q = clamp(trunc(x/scale +- 0.5), -127, 127) (the +-0.5 is an fp32 add). */
void rbo_quant_rows_v1(const float* x, int64_t rows, int64_t cols, int8_t* q, float* scale) {
    for (int64_t r = 0; r < rows; ++r) {
        const float* xr = x + r * cols;
        float amax = 0.0f;
        for (int64_t k = 0; k < cols; ++k) amax = fmaxf(amax, fabsf(xr[k]));
        float s = fmaxf(amax / 127.0f, 1e-8f);
        for (int64_t k = 0; k < cols; ++k) {
            float v = xr[k] / s;
            v = (v >= 0.0f) ? (v + 0.5f) : (v - 0.5f);
            int32_t t = (int32_t)v; /* truncation toward zero */
            if (t < -127) t = -127;
            if (t > 127) t = 127;
            q[r * cols + k] = (int8_t)t;
        }
        scale[r] = s;
    }
}

/* ------------------------------------------------------------------ GEMM */
/* C[m,n] = sum_k A[m,k] * B[n,k]  (A row-major [M,K], B row-major [N,K]). */
void rbo_gemm_i8_i32(const int8_t* a, const int8_t* b, int64_t M, int64_t N, int64_t K, int32_t* c) {
    for (int64_t m = 0; m < M; ++m) {
        const int8_t* ar = a + m * K;
        for (int64_t n = 0; n < N; ++n) {
            const int8_t* br = b + n * K;
            int32_t acc = 0;
            for (int64_t k = 0; k < K; ++k) acc += (int32_t)ar[k] * (int32_t)br[k];
            c[m * N + n] = acc;
        }
    }
}

/* w8a8_triton_kernels.py:230-246 / kernels/quantization.py:94-99:
 * out = ((f32(acc) * sa) * sb[n]) + bias[n], each step one fp32 RN op,
 * then stored in out_dtype.  sa_per_row selects sa[m] vs sa[0]. */
void rbo_scaled_epilogue(const int32_t* acc, int64_t M, int64_t N, const float* sa, int sa_per_row,
                         const float* sb, const float* bias, int out_dtype, void* out) {
    for (int64_t m = 0; m < M; ++m) {
        float a = sa_per_row ? sa[m] : sa[0];
        for (int64_t n = 0; n < N; ++n) {
            float v = (float)acc[m * N + n];
            v = v * a;
            v = v * sb[n];
            if (bias) v = v + bias[n];
            store_elem(out, out_dtype, m * N + n, v);
        }
    }
}

/* -------------------------------------------------- whole RepEncoder row */
typedef struct {
    const void* table; int table_dtype; int64_t num_rows;
    const int64_t* const* values; const int64_t* const* offsets; const int64_t* nnz;
    int64_t n_slots, n_items, begin, end;
    const float* gamma; const float* beta; float eps; int act_mode; float static_scale;
    int8_t* q; float* scale; float* pooled_out; float* ln_out;
} rep_job;

static void* rep_worker(void* arg) {
    const rep_job* jb = (const rep_job*)arg;
    const int64_t D = 512, H = jb->n_slots * D;
    float* row = (float*)malloc(sizeof(float) * (size_t)H);
    float* y = (float*)malloc(sizeof(float) * (size_t)H);
    float* acc = (float*)malloc(sizeof(float) * (size_t)D);
    for (int64_t i = jb->begin; i < jb->end; ++i) {
        for (int64_t s = 0; s < jb->n_slots; ++s) {
            const int64_t* off = jb->offsets[s];
            const int64_t nz = jb->nnz[s];
            int64_t start = off[i];
            int64_t end = (i + 1 < jb->n_items) ? off[i + 1] : nz;
            if (start < 0) start = 0;
            if (start > nz) start = nz;
            if (end > nz) end = nz;
            for (int64_t d = 0; d < D; ++d) acc[d] = 0.0f;
            for (int64_t j = start; j < end; ++j) {
                int64_t id = jb->values[s][j];
                if (id < 0) id = 0;
                if (id > jb->num_rows - 1) id = jb->num_rows - 1;
                if (id == 0) continue;
                for (int64_t d = 0; d < D; ++d)
                    acc[d] = acc[d] + load_elem(jb->table, jb->table_dtype, id * D + d);
            }
            for (int64_t d = 0; d < D; ++d) row[s * D + d] = round_to(jb->table_dtype, acc[d]);
        }
        rbo_layernorm_row(row, jb->n_slots, jb->gamma, jb->beta, jb->eps, jb->table_dtype, y, NULL, NULL);
        if (jb->act_mode == 0) {
            rbo_quant_dynamic_v2(y, 1, H, jb->q + i * H, jb->scale + i);
        } else {
            rbo_quant_static_v2(y, H, jb->static_scale, jb->q + i * H);
        }
        if (jb->pooled_out) memcpy(jb->pooled_out + i * H, row, sizeof(float) * (size_t)H);
        if (jb->ln_out) memcpy(jb->ln_out + i * H, y, sizeof(float) * (size_t)H);
    }
    free(row);
    free(y);
    free(acc);
    return NULL;
}

/*
 * gather -> pool (table dtype) -> concat -> LayerNorm (row dtype = table
 * dtype) -> dynamic (act_mode 0) or static (act_mode 1) int8 quantisation.
 * values/offsets/nnz are per-slot arrays.  Optional outputs pooled/ln
 * receive fp32 copies of the row-dtype intermediates [N, S*512].  Items are
 * split over n_threads POSIX threads; results do not depend on n_threads.
 */
void rbo_rep_forward(const void* table, int table_dtype, int64_t num_rows,
                     const int64_t* const* values, const int64_t* const* offsets, const int64_t* nnz,
                     int64_t n_slots, int64_t n_items, const float* gamma, const float* beta, float eps,
                     int act_mode, float static_scale, int8_t* q, float* scale,
                     float* pooled_out, float* ln_out, int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    pthread_t th[256];
    rep_job jobs[256];
    int64_t chunk = (n_items + n_threads - 1) / n_threads;
    int started = 0;
    for (int t = 0; t < n_threads; ++t) {
        rep_job jb = {table, table_dtype, num_rows, values, offsets, nnz, n_slots, n_items,
                      t * chunk, (t + 1) * chunk, gamma, beta, eps, act_mode, static_scale,
                      q, scale, pooled_out, ln_out};
        if (jb.begin > n_items) jb.begin = n_items;
        if (jb.end > n_items) jb.end = n_items;
        jobs[t] = jb;
    }
    for (int t = 1; t < n_threads; ++t) {
        if (pthread_create(&th[t], NULL, rep_worker, &jobs[t]) == 0) {
            started = t;
        } else {
            rep_worker(&jobs[t]);
            th[t] = 0;
        }
    }
    rep_worker(&jobs[0]);
    for (int t = 1; t <= started; ++t)
        if (th[t]) pthread_join(th[t], NULL);
}
