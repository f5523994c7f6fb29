// quant.cu -- standalone int8 quantisers, weight quantisation and weight
// repacking (sm_100a).  All are HBM-bound row/element kernels: one CTA per
// row for the per-row quantisers (the row is read twice, the second time
// from L2), a grid-stride loop for the per-tensor one.
//
//   dynamic_quant_kernel  quantization/w8a8_triton_kernels.py:41-64
//   static_quant_kernel   quantization/w8a8_triton_kernels.py:23-38
//   rows_v1_quant_kernel  kernels/quantization.py:6-35
//   weight_quant_kernel   quantization/w8a8_preprocess.py:46-57
//   pack_nk_kernel        qweight_t [K,N] (any strides) -> [N,K] K-contiguous
#include "common.cuh"

namespace rb {

constexpr int kRowThreads = 256;

__device__ __forceinline__ float block_max(float v, float* smem) {
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, d));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) smem[warp] = v;
  __syncthreads();
  float m = 0.0f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, smem[w]);
  __syncthreads();
  return m;
}

// amax over a row of K elements of dtype DT (any alignment)
template <int DT>
__device__ __forceinline__ float row_absmax(const void* x, int64_t K) {
  float m = 0.0f;
  for (int64_t k = threadIdx.x; k < K; k += blockDim.x) m = fmaxf(m, fabsf(load_as_f32(x, DT, k)));
  return m;
}

template <int DT>
__global__ void __launch_bounds__(kRowThreads) dynamic_quant_kernel(const void* x, int64_t K, int64_t ldx,
                                                                     int8_t* q, int64_t ldq, float* scale) {
  __shared__ float red[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  const char* xr = reinterpret_cast<const char*>(x) + row * ldx * (DT == RB_F32 ? 4 : 2);
  float amax = block_max(row_absmax<DT>(xr, K), red);
  amax = fmaxf(amax, 1e-8f);
  const float inv = __fdiv_rn(127.0f, amax);
  int8_t* qr = q + row * ldq;
  for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
    float r = roundf(__fmul_rn(load_as_f32(xr, DT, k), inv));
    qr[k] = (int8_t)(int)fminf(fmaxf(r, -128.0f), 127.0f);
  }
  if (threadIdx.x == 0) scale[row] = __fdiv_rn(amax, 127.0f);
}

template <int DT>
__global__ void __launch_bounds__(kRowThreads) rows_v1_quant_kernel(const void* x, int64_t K, int64_t ldx,
                                                                     int8_t* q, int64_t ldq, float* scale) {
  __shared__ float red[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  const char* xr = reinterpret_cast<const char*>(x) + row * ldx * (DT == RB_F32 ? 4 : 2);
  const float amax = block_max(row_absmax<DT>(xr, K), red);
  const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-8f);
  int8_t* qr = q + row * ldq;
  for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
    float v = __fdiv_rn(load_as_f32(xr, DT, k), s);
    v = (v >= 0.0f) ? __fadd_rn(v, 0.5f) : __fsub_rn(v, 0.5f);
    int t = __float2int_rz(v);
    t = min(max(t, -127), 127);
    qr[k] = (int8_t)t;
  }
  if (threadIdx.x == 0) scale[row] = s;
}

template <int DT>
__global__ void static_quant_kernel(const void* x, int64_t n, const void* scale, int scale_dtype, int8_t* q) {
  const float inv = __fdiv_rn(1.0f, load_as_f32(scale, scale_dtype, 0));
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float r = roundf(__fmul_rn(load_as_f32(x, DT, i), inv));
    q[i] = (int8_t)(int)fminf(fmaxf(r, -128.0f), 127.0f);
  }
}

// quantize_weight_per_channel: amax over the row, clamp 1e-8, scale = amax/127,
// q = clamp(round_half_even(w / scale), -128, 127)  (torch.round is half-to-even)
template <int DT>
__global__ void __launch_bounds__(kRowThreads) weight_quant_kernel(const void* w, int64_t K, int64_t ldw,
                                                                   int8_t* q, float* scale) {
  __shared__ float red[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  const char* wr = reinterpret_cast<const char*>(w) + row * ldw * (DT == RB_F32 ? 4 : 2);
  float amax = block_max(row_absmax<DT>(wr, K), red);
  amax = fmaxf(amax, 1e-8f);
  const float s = __fdiv_rn(amax, 127.0f);
  int8_t* qr = q + row * K;
  for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
    float r = rintf(__fdiv_rn(load_as_f32(wr, DT, k), s));
    qr[k] = (int8_t)(int)fminf(fmaxf(r, -128.0f), 127.0f);
  }
  if (threadIdx.x == 0) scale[row] = s;
}

// dst[n*K + k] = src[k*stride_k + n*stride_n], 32x32 tiles through shared memory
__global__ void pack_nk_kernel(const int8_t* src, int64_t K, int64_t N, int64_t sk, int64_t sn, int8_t* dst) {
  __shared__ int8_t tile[32][33];
  const int64_t k0 = (int64_t)blockIdx.x * 32, n0 = (int64_t)blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t k = k0 + i, n = n0 + threadIdx.x;
    if (k < K && n < N) tile[i][threadIdx.x] = src[k * sk + n * sn];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t n = n0 + i, k = k0 + threadIdx.x;
    if (k < K && n < N) dst[n * K + k] = tile[threadIdx.x][i];
  }
}

static bool float_dtype(int dt) { return dt == RB_F32 || dt == RB_BF16 || dt == RB_F16; }

}  // namespace rb

using namespace rb;

static int check_rows(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, const int8_t* q,
                      int64_t ldq, const float* scale) {
  if (!float_dtype(x_dtype)) return fail(RB_ERR_VALUE, "x dtype must be f32/bf16/f16");
  if (M < 0 || K < 0) return fail(RB_ERR_VALUE, "negative shape");
  if (M > 0x7fffffffLL) return fail(RB_ERR_UNSUPPORTED, "more than 2^31-1 rows");
  if (M > 0 && (x == nullptr || q == nullptr || scale == nullptr)) return fail(RB_ERR_VALUE, "null pointer");
  if (ldx < K || ldq < K) return fail(RB_ERR_VALUE, "row stride smaller than K");
  return RB_OK;
}

#define RB_ROW_LAUNCH(KERNEL, DT, ...)                                                        \
  do {                                                                                        \
    if ((DT) == RB_BF16) KERNEL<RB_BF16><<<grid, kRowThreads, 0, st>>>(__VA_ARGS__);          \
    else if ((DT) == RB_F16) KERNEL<RB_F16><<<grid, kRowThreads, 0, st>>>(__VA_ARGS__);       \
    else KERNEL<RB_F32><<<grid, kRowThreads, 0, st>>>(__VA_ARGS__);                           \
  } while (0)

extern "C" int rb_quant_dynamic_per_token(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx,
                                          int8_t* q, int64_t ldq, float* scale, void* stream) {
  int rc = check_rows(x, x_dtype, M, K, ldx, q, ldq, scale);
  if (rc || M == 0) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  dim3 grid((unsigned)M);
  RB_ROW_LAUNCH(dynamic_quant_kernel, x_dtype, x, K, ldx, q, ldq, scale);
  return check_cuda(cudaGetLastError(), "dynamic_quant_kernel launch");
}

extern "C" int rb_quant_rows_v1(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int8_t* q,
                                int64_t ldq, float* scale, void* stream) {
  int rc = check_rows(x, x_dtype, M, K, ldx, q, ldq, scale);
  if (rc || M == 0) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  dim3 grid((unsigned)M);
  RB_ROW_LAUNCH(rows_v1_quant_kernel, x_dtype, x, K, ldx, q, ldq, scale);
  return check_cuda(cudaGetLastError(), "rows_v1_quant_kernel launch");
}

extern "C" int rb_quantize_weight_per_channel(const void* w, int w_dtype, int64_t N, int64_t K, int64_t ldw,
                                              int8_t* q, float* scale, void* stream) {
  int rc = check_rows(w, w_dtype, N, K, ldw, q, K, scale);
  if (rc || N == 0) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  dim3 grid((unsigned)N);
  RB_ROW_LAUNCH(weight_quant_kernel, w_dtype, w, K, ldw, q, scale);
  return check_cuda(cudaGetLastError(), "weight_quant_kernel launch");
}

extern "C" int rb_quant_static(const void* x, int x_dtype, int64_t numel, const void* scale, int scale_dtype,
                               int8_t* q, void* stream) {
  if (!float_dtype(x_dtype) || !float_dtype(scale_dtype)) return fail(RB_ERR_VALUE, "x/scale dtype must be f32/bf16/f16");
  if (numel < 0) return fail(RB_ERR_VALUE, "negative numel");
  if (numel == 0) return RB_OK;
  if (x == nullptr || q == nullptr || scale == nullptr) return fail(RB_ERR_VALUE, "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const int threads = 256;
  int64_t blocks = (numel + threads - 1) / threads;
  const int64_t cap = (int64_t)sm_count() * 8;
  dim3 grid((unsigned)(blocks < cap ? blocks : cap));
  if (x_dtype == RB_BF16) static_quant_kernel<RB_BF16><<<grid, threads, 0, st>>>(x, numel, scale, scale_dtype, q);
  else if (x_dtype == RB_F16) static_quant_kernel<RB_F16><<<grid, threads, 0, st>>>(x, numel, scale, scale_dtype, q);
  else static_quant_kernel<RB_F32><<<grid, threads, 0, st>>>(x, numel, scale, scale_dtype, q);
  return check_cuda(cudaGetLastError(), "static_quant_kernel launch");
}

extern "C" int rb_pack_weight_nk(const int8_t* src, int64_t K, int64_t N, int64_t stride_k, int64_t stride_n,
                                 int8_t* dst, void* stream) {
  if (K < 0 || N < 0) return fail(RB_ERR_VALUE, "negative shape");
  if (K == 0 || N == 0) return RB_OK;
  if (src == nullptr || dst == nullptr) return fail(RB_ERR_VALUE, "null pointer");
  if ((K + 31) / 32 > 0x7fffffffLL || (N + 31) / 32 > 65535) return fail(RB_ERR_UNSUPPORTED, "weight too large");
  dim3 grid((unsigned)((K + 31) / 32), (unsigned)((N + 31) / 32)), block(32, 8);
  pack_nk_kernel<<<grid, block, 0, (cudaStream_t)stream>>>(src, K, N, stride_k, stride_n, dst);
  return check_cuda(cudaGetLastError(), "pack_nk_kernel launch");
}
