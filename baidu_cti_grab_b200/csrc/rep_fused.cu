// rep_fused.cu -- K1: fused embedding-bag gather -> fp32 sum-pool -> concat ->
// LayerNorm -> int8 quantisation for the RepEncoder (sm_100a).
//
// Replaces, in one launch per batch, the reference's
//   models.py:27-34   28x (values.clamp(0, V-1); nn.EmbeddingBag(sum, padding_idx=0))
//   models.py:39-45   torch.cat(..., dim=1) + nn.LayerNorm(28*512)
//   quantization/w8a8_triton_kernels.py:41-64 / 23-38  dynamic / static int8 quantiser
// The concatenated [N, 14336] row never reaches HBM: one CTA owns one item,
// warp w owns slots 4w..4w+3, and lane l of a warp owns columns 8l..8l+7 and
// 256+8l..256+8l+7 of each of its slots (two 16-byte vectors of a bf16 row).
// Those values stay in registers through the three LayerNorm passes and the
// quantiser.  Statistics use the fixed ("canonical") reduction order stated in
// the oracle: lane partials in column order, xor-butterfly 16..1 across the
// warp, slot totals in slot order.  Every floating-point step is an explicit
// round-to-nearest intrinsic so the result is reproducible bit for bit.
//
// HBM traffic per item (bf16 table, k ids per slot): 28*k*1 KB of table rows
// + 28*k*8 B ids + 28*2*8 B offsets + 14336 B int8 + 4 B scale.
#include "common.cuh"

namespace rb {

constexpr int kSlotsPerWarp = 4;
constexpr int kDim = 512;
constexpr int kRowsInFlight = 4;  // table rows a warp keeps in flight

enum RepMode : int { kGatherLnQuant = 0, kGatherPool = 1, kDenseLnQuant = 2 };

struct SlotArgs {
  const int64_t* values[RB_MAX_SLOTS];
  const int64_t* offsets[RB_MAX_SLOTS];
  int64_t nnz[RB_MAX_SLOTS];
  int col_slot[RB_MAX_SLOTS];
};

struct RepParams {
  SlotArgs slots;
  const void* table;
  int64_t num_rows;
  const void* x;  // dense pooled rows (kDenseLnQuant)
  int64_t ldx;
  int num_slots;
  int64_t num_items;
  const void* gamma;
  const void* beta;
  int ln_dtype;
  float eps;
  int act_mode;
  const void* static_scale;
  int static_scale_dtype;
  int8_t* q;
  int64_t ldq;
  float* scale;
  void* pooled;
  int64_t ldp;
  void* ln;
};

// 16 values of one slot held by one lane, in the row dtype.
template <typename T>
struct Frag;

template <>
struct Frag<__nv_bfloat16> {
  uint32_t w[8];  // w[0..3]: cols 8l..8l+7, w[4..7]: cols 256+8l..256+8l+7 (lo half first)
  __device__ __forceinline__ float get(int e) const {
    uint32_t v = w[e >> 1];
    return (e & 1) ? bf16_hi(v) : bf16_lo(v);
  }
  // store fp32 values rounded to bf16 (RNE)
  __device__ __forceinline__ void set_pair(int p, float lo, float hi) { w[p] = pack_bf16x2(lo, hi); }
  __device__ __forceinline__ void load(const void* row_base, int lane) {
    const uint4* p = reinterpret_cast<const uint4*>(row_base);
    uint4 a = p[lane], b = p[32 + lane];
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
    w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
  }
  __device__ __forceinline__ void store(void* row_base, int lane) const {
    uint4* p = reinterpret_cast<uint4*>(row_base);
    p[lane] = make_uint4(w[0], w[1], w[2], w[3]);
    p[32 + lane] = make_uint4(w[4], w[5], w[6], w[7]);
  }
};

template <>
struct Frag<float> {
  float f[16];
  __device__ __forceinline__ float get(int e) const { return f[e]; }
  __device__ __forceinline__ void set_pair(int p, float lo, float hi) {
    f[2 * p] = lo;
    f[2 * p + 1] = hi;
  }
  __device__ __forceinline__ void load(const void* row_base, int lane) {
    const float4* p = reinterpret_cast<const float4*>(row_base);
    float4 a = p[2 * lane], b = p[2 * lane + 1], c = p[64 + 2 * lane], d = p[64 + 2 * lane + 1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    f[8] = c.x; f[9] = c.y; f[10] = c.z; f[11] = c.w; f[12] = d.x; f[13] = d.y; f[14] = d.z; f[15] = d.w;
  }
  __device__ __forceinline__ void store(void* row_base, int lane) const {
    float4* p = reinterpret_cast<float4*>(row_base);
    p[2 * lane] = make_float4(f[0], f[1], f[2], f[3]);
    p[2 * lane + 1] = make_float4(f[4], f[5], f[6], f[7]);
    p[64 + 2 * lane] = make_float4(f[8], f[9], f[10], f[11]);
    p[64 + 2 * lane + 1] = make_float4(f[12], f[13], f[14], f[15]);
  }
};

// Raw table row piece of one lane (same column ownership as Frag).
template <typename T>
struct RowBuf;

template <>
struct RowBuf<__nv_bfloat16> {
  uint4 a, b;
  __device__ __forceinline__ void load(const __nv_bfloat16* row, int lane) {
    const uint4* p = reinterpret_cast<const uint4*>(row);
    a = __ldg(p + lane);
    b = __ldg(p + 32 + lane);
  }
  __device__ __forceinline__ void add_to(float* acc) const {
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      acc[2 * i] = __fadd_rn(acc[2 * i], bf16_lo(w[i]));
      acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], bf16_hi(w[i]));
    }
  }
};

template <>
struct RowBuf<float> {
  float4 a, b, c, d;
  __device__ __forceinline__ void load(const float* row, int lane) {
    const float4* p = reinterpret_cast<const float4*>(row);
    a = __ldg(p + 2 * lane);
    b = __ldg(p + 2 * lane + 1);
    c = __ldg(p + 64 + 2 * lane);
    d = __ldg(p + 64 + 2 * lane + 1);
  }
  __device__ __forceinline__ void add_to(float* acc) const {
    const float v[16] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w,
                         c.x, c.y, c.z, c.w, d.x, d.y, d.z, d.w};
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = __fadd_rn(acc[i], v[i]);
  }
};

// 8 consecutive LayerNorm affine parameters, widened to fp32.
__device__ __forceinline__ void load8_f32(const void* p, int dtype, int64_t idx, float* out) {
  if (dtype == RB_F32) {
    const float4* q = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + idx);
    float4 a = __ldg(q), b = __ldg(q + 1);
    out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
    out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
  } else {
    uint4 v = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p) + idx));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (dtype == RB_BF16) {
        out[2 * i] = bf16_lo(w[i]);
        out[2 * i + 1] = bf16_hi(w[i]);
      } else {
        __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
        float2 f = __half22float2(h);
        out[2 * i] = f.x;
        out[2 * i + 1] = f.y;
      }
    }
  }
}

__device__ __forceinline__ float warp_sum_butterfly(float v) {
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, d));
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, d));
  return v;
}

// a[j] for a runtime j in [0, 4) without dynamic register indexing
__device__ __forceinline__ int64_t sel4(const int64_t* a, int j) {
  return j == 0 ? a[0] : (j == 1 ? a[1] : (j == 2 ? a[2] : a[3]));
}

__device__ __forceinline__ int64_t shfl_i64(int64_t v, int src) {
  int lo = __shfl_sync(0xffffffffu, (int)(v & 0xffffffff), src);
  int hi = __shfl_sync(0xffffffffu, (int)(v >> 32), src);
  return ((int64_t)hi << 32) | (uint32_t)lo;
}

template <typename T, int MODE>
__global__ void __launch_bounds__(256, 2) rep_fused_kernel(const __grid_constant__ RepParams p) {
  __shared__ float s_tot[RB_MAX_SLOTS];
  __shared__ float s_wmax[8];
  __shared__ float s_stat[4];  // mean, rstd, scale, inv

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t item = blockIdx.x;
  const int S = p.num_slots;
  const int slot0 = warp * kSlotsPerWarp;
  const int nsl = max(0, min(kSlotsPerWarp, S - slot0));

  Frag<T> frag[kSlotsPerWarp];

  if constexpr (MODE == kDenseLnQuant) {
    const T* xrow = reinterpret_cast<const T*>(p.x) + item * p.ldx;
#pragma unroll
    for (int j = 0; j < kSlotsPerWarp; ++j)
      if (j < nsl) frag[j].load(xrow + (int64_t)(slot0 + j) * kDim, lane);
  } else {
    // ---- bag bounds of this warp's slots: lanes 0-3 starts, lanes 4-7 ends
    int64_t bound = 0;
    {
      const int j = lane & 3;
      if (lane < 8 && j < nsl) {
        const int s = slot0 + j;
        const int64_t nz = p.slots.nnz[s];
        const int64_t* off = p.slots.offsets[s];
        int64_t b;
        if (lane < 4) {
          b = off[item];
        } else {
          b = (item + 1 < p.num_items) ? off[item + 1] : nz;
        }
        bound = b < 0 ? 0 : (b > nz ? nz : b);
      }
    }
    int64_t start[kSlotsPerWarp], cnt[kSlotsPerWarp];
    int64_t total = 0, pre[kSlotsPerWarp + 1];
#pragma unroll
    for (int j = 0; j < kSlotsPerWarp; ++j) {
      start[j] = shfl_i64(bound, j);
      const int64_t e = shfl_i64(bound, 4 + j);
      cnt[j] = (j < nsl && e > start[j]) ? e - start[j] : 0;
      pre[j] = total;
      total += cnt[j];
    }
    pre[kSlotsPerWarp] = total;

    const T* table = reinterpret_cast<const T*>(p.table);
    const int64_t vmax = p.num_rows - 1;
    float acc[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) acc[e] = 0.0f;
    int cur = 0;  // slot (0..nsl) whose bag is being summed

    auto finish_slot = [&](int j) {
      // round the fp32 bag sum to the row dtype (nn.EmbeddingBag output)
#pragma unroll
      for (int jj = 0; jj < kSlotsPerWarp; ++jj) {
        if (jj == j) {
#pragma unroll
          for (int pr = 0; pr < 8; ++pr) frag[jj].set_pair(pr, acc[2 * pr], acc[2 * pr + 1]);
        }
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) acc[e] = 0.0f;
    };

    for (int64_t w0 = 0; w0 < total; w0 += 32) {
      // ids of positions w0 .. w0+31 of the concatenated bag list
      int64_t my_id = 0;
      {
        const int64_t t = w0 + lane;
        if (t < total) {
          const int j = (t >= pre[1]) + (t >= pre[2]) + (t >= pre[3]);
          int64_t id = p.slots.values[slot0 + j][sel4(start, j) + (t - sel4(pre, j))];
          id = id < 0 ? 0 : (id > vmax ? vmax : id);
          my_id = id;
        }
      }
      const int nwin = (total - w0 < 32) ? (int)(total - w0) : 32;
      for (int u0 = 0; u0 < nwin; u0 += kRowsInFlight) {
        RowBuf<T> buf[kRowsInFlight];
        int64_t ids[kRowsInFlight];
#pragma unroll
        for (int u = 0; u < kRowsInFlight; ++u) {
          ids[u] = shfl_i64(my_id, (u0 + u) & 31);
          if (u0 + u < nwin && ids[u] != 0) buf[u].load(table + ids[u] * kDim, lane);
        }
#pragma unroll
        for (int u = 0; u < kRowsInFlight; ++u) {
          if (u0 + u < nwin) {
            const int64_t t = w0 + u0 + u;
            const int j = (t >= pre[1]) + (t >= pre[2]) + (t >= pre[3]);
            while (cur < j) {
              finish_slot(cur);
              ++cur;
            }
            if (ids[u] != 0) buf[u].add_to(acc);  // padding_idx 0 is excluded
          }
        }
      }
    }
    while (cur < nsl) {
      finish_slot(cur);
      ++cur;
    }

    if constexpr (MODE == kGatherPool) {
#pragma unroll
      for (int j = 0; j < kSlotsPerWarp; ++j) {
        if (j < nsl) {
          T* dst = reinterpret_cast<T*>(p.pooled) + item * p.ldp +
                   (int64_t)p.slots.col_slot[slot0 + j] * kDim;
          frag[j].store(dst, lane);
        }
      }
      return;
    } else {
      if (p.pooled != nullptr) {
#pragma unroll
        for (int j = 0; j < kSlotsPerWarp; ++j)
          if (j < nsl)
            frag[j].store(reinterpret_cast<T*>(p.pooled) + item * p.ldp + (int64_t)(slot0 + j) * kDim,
                          lane);
      }
    }
  }

  if constexpr (MODE != kGatherPool) {
    const float H = (float)(S * kDim);
    // ---- pass 1: mean
#pragma unroll
    for (int j = 0; j < kSlotsPerWarp; ++j) {
      if (j < nsl) {
        float a = 0.0f;
#pragma unroll
        for (int e = 0; e < 16; ++e) a = __fadd_rn(a, frag[j].get(e));
        a = warp_sum_butterfly(a);
        if (lane == 0) s_tot[slot0 + j] = a;
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.0f;
      for (int s = 0; s < S; ++s) t = __fadd_rn(t, s_tot[s]);
      s_stat[0] = __fdiv_rn(t, H);
    }
    __syncthreads();
    const float mean = s_stat[0];
    // ---- pass 2: variance (two-pass)
#pragma unroll
    for (int j = 0; j < kSlotsPerWarp; ++j) {
      if (j < nsl) {
        float a = 0.0f;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float d = __fsub_rn(frag[j].get(e), mean);
          a = __fmaf_rn(d, d, a);
        }
        a = warp_sum_butterfly(a);
        if (lane == 0) s_tot[slot0 + j] = a;
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.0f;
      for (int s = 0; s < S; ++s) t = __fadd_rn(t, s_tot[s]);
      const float var = __fdiv_rn(t, H);
      s_stat[1] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, p.eps)));
    }
    __syncthreads();
    const float rstd = s_stat[1];
    // ---- pass 3: normalise + affine, round to the row dtype, absmax
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < kSlotsPerWarp; ++j) {
      if (j < nsl) {
        const int64_t col0 = (int64_t)(slot0 + j) * kDim + 8 * lane;
        float g[16], b[16];
        load8_f32(p.gamma, p.ln_dtype, col0, g);
        load8_f32(p.gamma, p.ln_dtype, col0 + 256, g + 8);
        load8_f32(p.beta, p.ln_dtype, col0, b);
        load8_f32(p.beta, p.ln_dtype, col0 + 256, b + 8);
#pragma unroll
        for (int pr = 0; pr < 8; ++pr) {
          float y0 = __fmaf_rn(__fmul_rn(rstd, __fsub_rn(frag[j].get(2 * pr), mean)), g[2 * pr], b[2 * pr]);
          float y1 = __fmaf_rn(__fmul_rn(rstd, __fsub_rn(frag[j].get(2 * pr + 1), mean)), g[2 * pr + 1],
                               b[2 * pr + 1]);
          frag[j].set_pair(pr, y0, y1);
        }
#pragma unroll
        for (int e = 0; e < 16; ++e) amax = fmaxf(amax, fabsf(frag[j].get(e)));
        if (p.ln != nullptr)
          frag[j].store(reinterpret_cast<T*>(p.ln) + item * (int64_t)(S * kDim) + (int64_t)(slot0 + j) * kDim,
                        lane);
      }
    }
    if (p.act_mode == RB_ACT_NONE) return;
    amax = warp_max(amax);
    if (lane == 0) s_wmax[warp] = amax;
    __syncthreads();
    if (threadIdx.x == 0) {
      float inv;
      if (p.act_mode == RB_ACT_DYNAMIC) {
        float m = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, s_wmax[w]);
        m = fmaxf(m, 1e-8f);
        s_stat[2] = __fdiv_rn(m, 127.0f);
        inv = __fdiv_rn(127.0f, m);
        p.scale[item] = s_stat[2];
      } else {
        inv = __fdiv_rn(1.0f, load_as_f32(p.static_scale, p.static_scale_dtype, 0));
      }
      s_stat[3] = inv;
    }
    __syncthreads();
    const float inv = s_stat[3];
    // ---- pass 4: int8 = clamp(roundf(y * inv), -128, 127)
#pragma unroll
    for (int j = 0; j < kSlotsPerWarp; ++j) {
      if (j < nsl) {
        int qv[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float r = roundf(__fmul_rn(frag[j].get(e), inv));
          r = fminf(fmaxf(r, -128.0f), 127.0f);
          qv[e] = (int)r;
        }
        int8_t* dst = p.q + item * p.ldq + (int64_t)(slot0 + j) * kDim + 8 * lane;
        *reinterpret_cast<uint2*>(dst) =
            make_uint2(pack_i8x4(qv[0], qv[1], qv[2], qv[3]), pack_i8x4(qv[4], qv[5], qv[6], qv[7]));
        *reinterpret_cast<uint2*>(dst + 256) = make_uint2(pack_i8x4(qv[8], qv[9], qv[10], qv[11]),
                                                          pack_i8x4(qv[12], qv[13], qv[14], qv[15]));
      }
    }
  }
}

// ------------------------------------------------------------------ host
static int validate_common(int num_slots, int64_t num_items) {
  if (num_slots < 1 || num_slots > RB_MAX_SLOTS)
    return fail(RB_ERR_VALUE, "num_slots must be in [1, %d], got %d", RB_MAX_SLOTS, num_slots);
  if (num_items < 0) return fail(RB_ERR_VALUE, "num_items must be >= 0");
  if (num_items > 0x7fffffffLL) return fail(RB_ERR_UNSUPPORTED, "num_items above 2^31-1 per call");
  return RB_OK;
}

static int fill_slots(SlotArgs& sa, const int64_t* const* values, const int64_t* const* offsets,
                      const int64_t* nnz, const int* col_slot, int num_slots, int64_t num_items) {
  for (int s = 0; s < num_slots; ++s) {
    if (offsets == nullptr || offsets[s] == nullptr)
      return fail(RB_ERR_VALUE, "slot %d: offsets pointer is null", s);
    if (nnz[s] < 0) return fail(RB_ERR_VALUE, "slot %d: nnz must be >= 0", s);
    if (nnz[s] > 0 && (values == nullptr || values[s] == nullptr))
      return fail(RB_ERR_VALUE, "slot %d: values pointer is null", s);
    sa.values[s] = values ? values[s] : nullptr;
    sa.offsets[s] = offsets[s];
    sa.nnz[s] = nnz[s];
    sa.col_slot[s] = col_slot ? col_slot[s] : s;
  }
  (void)num_items;
  return RB_OK;
}

template <int MODE>
static int launch_rep(const RepParams& p, int row_dtype, cudaStream_t stream) {
  if (p.num_items == 0) return RB_OK;
  const int warps = (p.num_slots + kSlotsPerWarp - 1) / kSlotsPerWarp;
  dim3 grid((unsigned)p.num_items), block(32 * warps);
  if (row_dtype == RB_BF16)
    rep_fused_kernel<__nv_bfloat16, MODE><<<grid, block, 0, stream>>>(p);
  else
    rep_fused_kernel<float, MODE><<<grid, block, 0, stream>>>(p);
  return check_cuda(cudaGetLastError(), "rep_fused_kernel launch");
}

static int check_ln_args(const void* gamma, const void* beta, int ln_dtype, int act_mode,
                         const void* static_scale, int ss_dtype, const int8_t* q, int64_t ldq,
                         const float* scale, const void* ln_out, int num_slots) {
  if (gamma == nullptr || beta == nullptr) return fail(RB_ERR_VALUE, "LayerNorm gamma/beta must be given");
  if (ln_dtype != RB_BF16 && ln_dtype != RB_F32 && ln_dtype != RB_F16)
    return fail(RB_ERR_VALUE, "ln_dtype must be RB_BF16, RB_F16 or RB_F32");
  if (!aligned(gamma, 16) || !aligned(beta, 16)) return fail(RB_ERR_VALUE, "gamma/beta must be 16-byte aligned");
  if (act_mode == RB_ACT_DYNAMIC || act_mode == RB_ACT_STATIC) {
    if (q == nullptr) return fail(RB_ERR_VALUE, "q_out must be given");
    if (!aligned(q, 16) || ldq % 16 != 0 || ldq < (int64_t)num_slots * kDim)
      return fail(RB_ERR_VALUE, "q_out must be 16-byte aligned with ldq %% 16 == 0 and ldq >= %d",
                  num_slots * kDim);
    if (act_mode == RB_ACT_DYNAMIC && scale == nullptr) return fail(RB_ERR_VALUE, "scale_out must be given");
    if (act_mode == RB_ACT_STATIC) {
      if (static_scale == nullptr) return fail(RB_ERR_VALUE, "static_scale must be given");
      if (ss_dtype != RB_F32 && ss_dtype != RB_BF16 && ss_dtype != RB_F16)
        return fail(RB_ERR_VALUE, "static_scale dtype must be f32/bf16/f16");
    }
  } else if (act_mode == RB_ACT_NONE) {
    if (ln_out == nullptr) return fail(RB_ERR_VALUE, "act_mode RB_ACT_NONE needs ln_out");
  } else {
    return fail(RB_ERR_VALUE, "unknown act_mode %d", act_mode);
  }
  if (ln_out != nullptr && !aligned(ln_out, 16)) return fail(RB_ERR_VALUE, "ln_out must be 16-byte aligned");
  return RB_OK;
}

}  // namespace rb

using namespace rb;

extern "C" int rb_rep_gather_ln_quant(const void* table, int table_dtype, int64_t num_rows, int emb_dim,
                                      const int64_t* const* slot_values, const int64_t* const* slot_offsets,
                                      const int64_t* slot_nnz, int num_slots, int64_t num_items,
                                      const void* ln_gamma, const void* ln_beta, int ln_dtype, float eps,
                                      int act_mode, const void* static_scale, int static_scale_dtype,
                                      int8_t* q_out, int64_t ldq, float* scale_out, void* pooled_out,
                                      void* ln_out, void* stream) {
  int rc = validate_common(num_slots, num_items);
  if (rc) return rc;
  if (emb_dim != kDim) return fail(RB_ERR_UNSUPPORTED, "emb_dim must be 512, got %d", emb_dim);
  if (table_dtype != RB_BF16 && table_dtype != RB_F32)
    return fail(RB_ERR_VALUE, "table dtype must be RB_BF16 or RB_F32");
  if (table == nullptr || !aligned(table, 16)) return fail(RB_ERR_VALUE, "table must be 16-byte aligned");
  if (num_rows < 1) return fail(RB_ERR_VALUE, "num_rows must be >= 1");
  if (slot_nnz == nullptr) return fail(RB_ERR_VALUE, "slot_nnz must be given");
  rc = check_ln_args(ln_gamma, ln_beta, ln_dtype, act_mode, static_scale, static_scale_dtype, q_out, ldq,
                     scale_out, ln_out, num_slots);
  if (rc) return rc;
  if (pooled_out != nullptr && !aligned(pooled_out, 16))
    return fail(RB_ERR_VALUE, "pooled_out must be 16-byte aligned");
  RepParams p{};
  rc = fill_slots(p.slots, slot_values, slot_offsets, slot_nnz, nullptr, num_slots, num_items);
  if (rc) return rc;
  p.table = table;
  p.num_rows = num_rows;
  p.num_slots = num_slots;
  p.num_items = num_items;
  p.gamma = ln_gamma;
  p.beta = ln_beta;
  p.ln_dtype = ln_dtype;
  p.eps = eps;
  p.act_mode = act_mode;
  p.static_scale = static_scale;
  p.static_scale_dtype = static_scale_dtype;
  p.q = q_out;
  p.ldq = ldq;
  p.scale = scale_out;
  p.pooled = pooled_out;
  p.ldp = (int64_t)num_slots * kDim;
  p.ln = ln_out;
  return launch_rep<kGatherLnQuant>(p, table_dtype, (cudaStream_t)stream);
}

extern "C" int rb_rep_gather_pool(const void* table, int table_dtype, int64_t num_rows, int emb_dim,
                                  const int64_t* const* slot_values, const int64_t* const* slot_offsets,
                                  const int64_t* slot_nnz, const int* col_slot, int num_slots,
                                  int64_t num_items, void* pooled_out, int64_t ldp, void* stream) {
  int rc = validate_common(num_slots, num_items);
  if (rc) return rc;
  if (emb_dim != kDim) return fail(RB_ERR_UNSUPPORTED, "emb_dim must be 512, got %d", emb_dim);
  if (table_dtype != RB_BF16 && table_dtype != RB_F32)
    return fail(RB_ERR_VALUE, "table dtype must be RB_BF16 or RB_F32");
  if (table == nullptr || !aligned(table, 16)) return fail(RB_ERR_VALUE, "table must be 16-byte aligned");
  if (num_rows < 1) return fail(RB_ERR_VALUE, "num_rows must be >= 1");
  if (slot_nnz == nullptr || col_slot == nullptr) return fail(RB_ERR_VALUE, "slot_nnz/col_slot must be given");
  if (pooled_out == nullptr || !aligned(pooled_out, 16))
    return fail(RB_ERR_VALUE, "pooled_out must be 16-byte aligned");
  const int esz = dtype_size(table_dtype);
  if ((ldp * esz) % 16 != 0) return fail(RB_ERR_VALUE, "ldp must keep rows 16-byte aligned");
  for (int s = 0; s < num_slots; ++s)
    if (col_slot[s] < 0 || (int64_t)(col_slot[s] + 1) * kDim > ldp)
      return fail(RB_ERR_VALUE, "col_slot[%d]=%d does not fit in ldp=%lld", s, col_slot[s], (long long)ldp);
  RepParams p{};
  rc = fill_slots(p.slots, slot_values, slot_offsets, slot_nnz, col_slot, num_slots, num_items);
  if (rc) return rc;
  p.table = table;
  p.num_rows = num_rows;
  p.num_slots = num_slots;
  p.num_items = num_items;
  p.pooled = pooled_out;
  p.ldp = ldp;
  return launch_rep<kGatherPool>(p, table_dtype, (cudaStream_t)stream);
}

extern "C" int rb_layernorm_quant(const void* x, int x_dtype, int64_t num_items, int num_slots, int64_t ldx,
                                  const void* ln_gamma, const void* ln_beta, int ln_dtype, float eps,
                                  int act_mode, const void* static_scale, int static_scale_dtype,
                                  int8_t* q_out, int64_t ldq, float* scale_out, void* ln_out, void* stream) {
  int rc = validate_common(num_slots, num_items);
  if (rc) return rc;
  if (x_dtype != RB_BF16 && x_dtype != RB_F32) return fail(RB_ERR_VALUE, "x dtype must be RB_BF16 or RB_F32");
  const int esz = dtype_size(x_dtype);
  if (x == nullptr || !aligned(x, 16) || (ldx * esz) % 16 != 0 || ldx < (int64_t)num_slots * kDim)
    return fail(RB_ERR_VALUE, "x must be 16-byte aligned with 16-byte row stride and ldx >= %d",
                num_slots * kDim);
  rc = check_ln_args(ln_gamma, ln_beta, ln_dtype, act_mode, static_scale, static_scale_dtype, q_out, ldq,
                     scale_out, ln_out, num_slots);
  if (rc) return rc;
  RepParams p{};
  p.x = x;
  p.ldx = ldx;
  p.num_slots = num_slots;
  p.num_items = num_items;
  p.gamma = ln_gamma;
  p.beta = ln_beta;
  p.ln_dtype = ln_dtype;
  p.eps = eps;
  p.act_mode = act_mode;
  p.static_scale = static_scale;
  p.static_scale_dtype = static_scale_dtype;
  p.q = q_out;
  p.ldq = ldq;
  p.scale = scale_out;
  p.ln = ln_out;
  return launch_rep<kDenseLnQuant>(p, x_dtype, (cudaStream_t)stream);
}
