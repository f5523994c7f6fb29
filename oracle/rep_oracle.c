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
 *   rbo_layernorm_stats     models.py:21,45 nn.LayerNorm(S*D, eps) over the
 *   rbo_layernorm_apply     concatenated row, as ATen's CUDA LayerNorm
 *                           computes it (order below).
 *   rbo_quant_dynamic_v2    quantization/w8a8_triton_kernels.py:41-64
 *   rbo_quant_static_v2     quantization/w8a8_triton_kernels.py:23-38
 *   rbo_quant_rows_v1       kernels/quantization.py:6-35
 *   rbo_gemm_i8_i32         quantization/w8a8_triton_kernels.py:67-171 (int32 acc)
 *   rbo_scaled_epilogue     quantization/w8a8_triton_kernels.py:230-246
 *   rbo_rep_pool_stats      models.py:24-45 gather -> pool -> concat and the
 *   rbo_rep_finish          LayerNorm statistics; then LayerNorm + w8a8_linear's
 *                           int8 quantiser once rstd is known (see below).
 *
 * LayerNorm order.  The reference's nn.LayerNorm runs ATen's CUDA kernel on
 * the GPU (PyTorch, not vendored by the reference: it pins torch 2.6.0, and
 * the tests here run 2.11.0; aten/src/ATen/native/cuda/layer_norm_kernel.cu,
 * vectorized_layer_norm_kernel -> compute_stats, taken for rows whose length
 * is a multiple of 4 with aligned buffers, which every RepEncoder row is).
 * Its published algorithm, restated:
 *   * 128 threads per row (4 warps of 32).  Thread t walks the 4-element
 *     groups g = t, t+128, t+256, ... (elements 4g..4g+3 in order) with
 *     Welford's online update, state (mean, m2, count) from zeros:
 *       delta = x - mean; count = count + 1; r = 1/count (IEEE);
 *       mean = fma(delta, r, mean); m2 = fma(delta, x - mean_new, m2)
 *   * each warp combines its 32 states by shuffle-down with distances
 *     16, 8, 4, 2, 1 (lane l takes lane l+d), combine(B = own, A = other):
 *       delta = B.mean - A.mean; n = A.count + B.count; c = 1/n (IEEE);
 *       nA = A.count*c; nB = B.count*c; mean = fma(nA, A.mean, nB*B.mean);
 *       m2 = fma(delta*delta*A.count, nB, A.m2 + B.m2)
 *   * warps 0,1 take warps 2,3, then warp 0 takes warp 1 (same combine);
 *   * var = m2 / H (IEEE); rstd = rsqrtf(var + eps);
 *   * y = fma(gamma, rstd * (x - mean), beta), rounded to the row dtype.
 * rsqrtf is CUDA's hardware reciprocal square root (within 2 ulp, and not
 * correctly rounded on about a quarter of inputs), so this file does not
 * compute it: rbo_rep_pool_stats returns fl(var + eps) per row and the caller
 * supplies rstd (evaluated on the GPU by the GPU tests; the CPU-only default
 * in oracle.py is the correctly rounded value, which matches the GPU's to
 * within 2 ulp).  With that one value supplied, mean, rstd and every output
 * element equal ATen CUDA's bit for bit (pinned by tests/golden/ln_aten_cuda.npz,
 * recorded from ATen on a B200 by tests/golden/gen_golden_aten_cuda.py).
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

/* --------------------------------------------- LayerNorm (ATen CUDA order) */
typedef struct { float mean, m2, count; } welford;

/* layer_norm_kernel.cu cuWelfordOnlineSum */
static inline welford welford_push(welford s, float x) {
    welford o;
    const float delta = x - s.mean;
    o.count = s.count + 1.0f;
    o.mean = fmaf(delta, 1.0f / o.count, s.mean);
    o.m2 = fmaf(delta, x - o.mean, s.m2);
    return o;
}

/* layer_norm_kernel.cu cuWelfordCombine(dataB = b, dataA = a) */
static inline welford welford_merge(welford b, welford a) {
    welford o;
    o.count = a.count + b.count;
    if (o.count > 0.0f) {
        const float delta = b.mean - a.mean;
        const float c = 1.0f / o.count;
        const float na = a.count * c, nb = b.count * c;
        o.mean = fmaf(na, a.mean, nb * b.mean);
        o.m2 = fmaf(delta * delta * a.count, nb, a.m2 + b.m2);
    } else {
        o.mean = 0.0f;
        o.m2 = 0.0f;
    }
    return o;
}

/*
 * Mean and fl(var + eps) of one row x[H] (H % 4 == 0) in ATen CUDA's order
 * (file header).  var_eps is the argument of the rsqrtf that gives rstd.
 */
void rbo_layernorm_stats(const float* x, int64_t H, float eps, float* mean_out, float* var_eps_out) {
    welford th[128], warp_state[4];
    const int64_t groups = H / 4;
    for (int t = 0; t < 128; ++t) {
        welford s = {0.0f, 0.0f, 0.0f};
        for (int64_t g = t; g < groups; g += 128)
            for (int e = 0; e < 4; ++e) s = welford_push(s, x[4 * g + e]);
        th[t] = s;
    }
    for (int w = 0; w < 4; ++w) {
        welford l[32], n[32];
        memcpy(l, th + 32 * w, sizeof(l));
        for (int d = 16; d >= 1; d >>= 1) {
            /* a lane past the warp reads its own state (shuffle-down semantics) */
            for (int i = 0; i < 32; ++i) n[i] = welford_merge(l[i], i + d < 32 ? l[i + d] : l[i]);
            memcpy(l, n, sizeof(l));
        }
        warp_state[w] = l[0];
    }
    warp_state[0] = welford_merge(warp_state[0], warp_state[2]);
    warp_state[1] = welford_merge(warp_state[1], warp_state[3]);
    warp_state[0] = welford_merge(warp_state[0], warp_state[1]);
    *mean_out = warp_state[0].mean;
    *var_eps_out = warp_state[0].m2 / (float)H + eps;
}

/* y[k] = round_to(out_dtype, fma(gamma[k], rstd * (x[k] - mean), beta[k])) */
void rbo_layernorm_apply(const float* x, int64_t H, float mean, float rstd, const float* gamma,
                         const float* beta, int out_dtype, float* y) {
    for (int64_t k = 0; k < H; ++k) y[k] = round_to(out_dtype, fmaf(gamma[k], rstd * (x[k] - mean), beta[k]));
}

/* Statistics of rows x[M, H]: mean[M] and fl(var + eps)[M]. */
void rbo_layernorm_stats_rows(const float* x, int64_t M, int64_t H, float eps, float* mean, float* var_eps) {
    for (int64_t r = 0; r < M; ++r) rbo_layernorm_stats(x + r * H, H, eps, mean + r, var_eps + r);
}

/* LayerNorm of rows x[M, H] given per-row mean and rstd. */
void rbo_layernorm_apply_rows(const float* x, int64_t M, int64_t H, const float* mean, const float* rstd,
                              const float* gamma, const float* beta, int out_dtype, float* y) {
    for (int64_t r = 0; r < M; ++r) rbo_layernorm_apply(x + r * H, H, mean[r], rstd[r], gamma, beta, out_dtype, y + r * H);
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
/* Items [begin, end) of a batch are split over POSIX threads; results do not
 * depend on the thread count. */
typedef struct {
    const void* table; int table_dtype; int64_t num_rows;
    const int64_t* const* values; const int64_t* const* offsets; const int64_t* nnz;
    int64_t n_slots, n_items, begin, end;
    float eps; float* pooled; float* mean; float* var_eps;
    const float* rstd; const float* gamma; const float* beta; int act_mode; float static_scale;
    int8_t* q; float* scale; float* ln_out;
} rep_job;

static void* pool_stats_worker(void* arg) {
    const rep_job* jb = (const rep_job*)arg;
    const int64_t D = 512, H = jb->n_slots * D;
    float* acc = (float*)malloc(sizeof(float) * (size_t)D);
    for (int64_t i = jb->begin; i < jb->end; ++i) {
        float* row = jb->pooled + i * H;
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
        rbo_layernorm_stats(row, H, jb->eps, jb->mean + i, jb->var_eps + i);
    }
    free(acc);
    return NULL;
}

static void* finish_worker(void* arg) {
    const rep_job* jb = (const rep_job*)arg;
    const int64_t H = jb->n_slots * 512;
    float* y = (float*)malloc(sizeof(float) * (size_t)H);
    for (int64_t i = jb->begin; i < jb->end; ++i) {
        rbo_layernorm_apply(jb->pooled + i * H, H, jb->mean[i], jb->rstd[i], jb->gamma, jb->beta,
                            jb->table_dtype, y);
        if (jb->act_mode == 0) {
            rbo_quant_dynamic_v2(y, 1, H, jb->q + i * H, jb->scale + i);
        } else {
            rbo_quant_static_v2(y, H, jb->static_scale, jb->q + i * H);
        }
        if (jb->ln_out) memcpy(jb->ln_out + i * H, y, sizeof(float) * (size_t)H);
    }
    free(y);
    return NULL;
}

static void run_jobs(rep_job proto, int n_threads, void* (*fn)(void*)) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    pthread_t th[256];
    rep_job jobs[256];
    int ok[256];
    const int64_t chunk = (proto.n_items + n_threads - 1) / n_threads;
    for (int t = 0; t < n_threads; ++t) {
        jobs[t] = proto;
        jobs[t].begin = t * chunk < proto.n_items ? t * chunk : proto.n_items;
        jobs[t].end = (t + 1) * chunk < proto.n_items ? (t + 1) * chunk : proto.n_items;
    }
    for (int t = 1; t < n_threads; ++t) {
        ok[t] = pthread_create(&th[t], NULL, fn, &jobs[t]) == 0;
        if (!ok[t]) fn(&jobs[t]);
    }
    fn(&jobs[0]);
    for (int t = 1; t < n_threads; ++t)
        if (ok[t]) pthread_join(th[t], NULL);
}

/*
 * models.py:24-45 up to the LayerNorm statistics: per item, gather + pool each
 * slot (fp32 in bag order, one round to the table dtype; models.py:27-33),
 * concatenate into pooled[i, S*512] (fp32 values of the row dtype; models.py:43)
 * and take the row's LayerNorm mean and fl(var + eps) in ATen CUDA's order.
 */
void rbo_rep_pool_stats(const void* table, int table_dtype, int64_t num_rows,
                        const int64_t* const* values, const int64_t* const* offsets, const int64_t* nnz,
                        int64_t n_slots, int64_t n_items, float eps, float* pooled, float* mean,
                        float* var_eps, int n_threads) {
    rep_job jb;
    memset(&jb, 0, sizeof(jb));
    jb.table = table; jb.table_dtype = table_dtype; jb.num_rows = num_rows;
    jb.values = values; jb.offsets = offsets; jb.nnz = nnz;
    jb.n_slots = n_slots; jb.n_items = n_items; jb.eps = eps;
    jb.pooled = pooled; jb.mean = mean; jb.var_eps = var_eps;
    run_jobs(jb, n_threads, pool_stats_worker);
}

/*
 * models.py:45 + w8a8_linear's quantiser: LayerNorm of the pooled rows with the
 * given mean and rstd (y rounded to the row dtype), then dynamic (act_mode 0)
 * or static (act_mode 1) int8 quantisation; ln_out (optional) receives y.
 */
void rbo_rep_finish(const float* pooled, int row_dtype, int64_t n_slots, int64_t n_items, const float* mean,
                    const float* rstd, const float* gamma, const float* beta, int act_mode, float static_scale,
                    int8_t* q, float* scale, float* ln_out, int n_threads) {
    rep_job jb;
    memset(&jb, 0, sizeof(jb));
    jb.table_dtype = row_dtype; jb.n_slots = n_slots; jb.n_items = n_items;
    jb.pooled = (float*)pooled; jb.mean = (float*)mean; jb.rstd = rstd;
    jb.gamma = gamma; jb.beta = beta; jb.act_mode = act_mode; jb.static_scale = static_scale;
    jb.q = q; jb.scale = scale; jb.ln_out = ln_out;
    run_jobs(jb, n_threads, finish_worker);
}
