// Quantisers feeding the INT8 / FP8-e4m3 tcgen05 projections.
//
// INT8 (the config-2 scheme, applied to qkv_proj, out_proj and to_out_linear):
//   scale_r = max(amax_r / 127, 1e-12) in fp32, q = round_half_even(x / scale_r) clamped
//   to [-127, 127], one scale per row.  Rows are tokens for activations and output
//   channels for weights, so the same kernel serves both.  Division is IEEE fp32, so the
//   codes match a CPU fp32 restatement bit for bit.
// FP8 e4m3 per tensor (fp8.py:99-133 with per_tensor=True, the sm>=100 rule of fp8.py:84-85):
//   scale = max(amax / 448, 1e-12), q = e4m3_rn(clamp(x / scale, -448, 448)).
#include "host_common.h"
#include "sm100.cuh"

namespace vdn {
namespace quant {

__device__ __forceinline__ float block_max(float v) {
  __shared__ float red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = (l < (int)(blockDim.x >> 5)) ? red[l] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (l == 0) red[0] = v;
  }
  __syncthreads();
  const float r = red[0];
  __syncthreads();
  return r;
}

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// one block per row
template <typename T>
__global__ void int8_rows_kernel(const T* __restrict__ x, long long ldx, int K, int8_t* __restrict__ q, long long ldq,
                                 float* __restrict__ scale) {
  const long long r = blockIdx.x;
  const T* row = x + r * ldx;
  float amax = 0.f;
  for (int c = threadIdx.x; c < K; c += blockDim.x) amax = fmaxf(amax, fabsf(to_f<T>(row[c])));
  amax = block_max(amax);
  const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-12f);
  if (threadIdx.x == 0) scale[r] = s;
  int8_t* qr = q + r * ldq;
  for (int c = threadIdx.x; c < K; c += blockDim.x) {
    float v = rintf(__fdiv_rn(to_f<T>(row[c]), s));
    v = fminf(fmaxf(v, -127.f), 127.f);
    qr[c] = static_cast<int8_t>(static_cast<int>(v));
  }
}

template <typename T>
__global__ void amax_kernel(const T* __restrict__ x, long long ldx, int rows, int K, float* __restrict__ amax) {
  float m = 0.f;
  const long long n = (long long)rows * K;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
    const long long r = e / K;
    const int c = (int)(e % K);
    m = fmaxf(m, fabsf(to_f<T>(x[r * ldx + c])));
  }
  m = block_max(m);
  if (threadIdx.x == 0) atomicMax(reinterpret_cast<int*>(amax), __float_as_int(m));
}

template <typename T>
__global__ void fp8_cast_kernel(const T* __restrict__ x, long long ldx, int rows, int K, const float* __restrict__ amax,
                                __nv_fp8_e4m3* __restrict__ q, long long ldq, float* __restrict__ scale_out) {
  const float s = fmaxf(__fdiv_rn(*amax, 448.0f), 1e-12f);
  if (blockIdx.x == 0 && threadIdx.x == 0 && scale_out) *scale_out = s;
  const long long n = (long long)rows * K;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
    const long long r = e / K;
    const int c = (int)(e % K);
    float v = __fdiv_rn(to_f<T>(x[r * ldx + c]), s);
    v = fminf(fmaxf(v, -448.f), 448.f);
    q[r * ldq + c] = __nv_fp8_e4m3(v);
  }
}

}  // namespace quant
}  // namespace vdn

extern "C" {

// Per-row symmetric int8.  src_kind 0 = bf16, 1 = fp32.  q [rows, ldq] int8, scale [rows] fp32.
int vdn_quant_int8_rows(int src_kind, const void* x, long long ldx, int rows, int K, void* q, long long ldq,
                        float* scale, void* stream) {
  if (!x || !q || !scale || rows < 0 || K <= 0) return vdn::kBadArgument;
  if (rows == 0) return vdn::kOk;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (src_kind == 0)
    vdn::quant::int8_rows_kernel<__nv_bfloat16><<<rows, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(x), ldx, K,
                                                                      reinterpret_cast<int8_t*>(q), ldq, scale);
  else
    vdn::quant::int8_rows_kernel<float><<<rows, 256, 0, s>>>(reinterpret_cast<const float*>(x), ldx, K,
                                                              reinterpret_cast<int8_t*>(q), ldq, scale);
  return vdn::launch_status();
}

// Per-tensor e4m3.  work: one fp32 device scalar (zeroed here) that receives the amax;
// scale_out: the fp32 dequantisation scale.  src_kind 0 = bf16, 1 = fp32.
int vdn_quant_fp8_tensor(int src_kind, const void* x, long long ldx, int rows, int K, void* q, long long ldq,
                         float* work, float* scale_out, void* stream) {
  if (!x || !q || !work || !scale_out || rows < 0 || K <= 0) return vdn::kBadArgument;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  cudaMemsetAsync(work, 0, sizeof(float), s);
  const long long n = (long long)rows * K;
  const int blocks = (int)std::min<long long>((n + 255) / 256, 4LL * vdn::sm_count());
  if (blocks > 0) {
    if (src_kind == 0) {
      vdn::quant::amax_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(x), ldx,
                                                                     rows, K, work);
      vdn::quant::fp8_cast_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(
          reinterpret_cast<const __nv_bfloat16*>(x), ldx, rows, K, work, reinterpret_cast<__nv_fp8_e4m3*>(q), ldq,
          scale_out);
    } else {
      vdn::quant::amax_kernel<float><<<blocks, 256, 0, s>>>(reinterpret_cast<const float*>(x), ldx, rows, K, work);
      vdn::quant::fp8_cast_kernel<float><<<blocks, 256, 0, s>>>(reinterpret_cast<const float*>(x), ldx, rows, K, work,
                                                                 reinterpret_cast<__nv_fp8_e4m3*>(q), ldq, scale_out);
    }
  }
  return vdn::launch_status();
}

}  // extern "C"
