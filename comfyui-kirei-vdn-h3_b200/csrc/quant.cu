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

// rint(x / s) for |x / s| <= 128, bit-identical to rintf(__fdiv_rn(x, s)), the x / scale of
// the CPU restatement.  r = 1/s correctly rounded, so q = x * r (both roundings included) lies
// within 128 * 2^-23 = 2^-16 of x / s, and the correctly rounded quotient within 2^-17 of it:
// the two round to the same integer unless q is within 2^-15 of a half-integer.  Elements with
// q within 2^-12 of one (about 1 in 2,000) take the IEEE division instead.  q - rint(q) is
// exact (Sterbenz), and __fmul_rn keeps the product from being fused into the subtraction.
__device__ __forceinline__ float rint_quotient(float x, float s, float r) {
  const float q = __fmul_rn(x, r);
  const float c = rintf(q);
  return fabsf(__fsub_rn(q, c)) <= 0.5f - 0x1p-12f ? c : rintf(__fdiv_rn(x, s));
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

// bf16 rows read once into registers with 16-byte loads (NV vectors of 8 per thread of
// THREADS, K <= 8 * THREADS * NV), same rule as int8_rows_kernel; codes stored 8 per 8-byte
// store.  Wide rows use more threads, not more registers, so several CTAs share an SM.
template <int NV, int THREADS>
__global__ void __launch_bounds__(THREADS) int8_rows_vec_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                             int K, int8_t* __restrict__ q, long long ldq,
                                                             float* __restrict__ scale) {
  const long long r = blockIdx.x;
  const uint4* row = reinterpret_cast<const uint4*>(x + r * ldx);
  const int nvec = K >> 3;
  uint4 v[NV];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int vi = threadIdx.x + THREADS * i;
    v[i] = vi < nvec ? __ldg(row + vi) : make_uint4(0, 0, 0, 0);
    const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
    for (int e = 0; e < 4; ++e)
      amax = fmaxf(amax, fmaxf(fabsf(__uint_as_float(w[e] << 16)), fabsf(__uint_as_float(w[e] & 0xFFFF0000u))));
  }
  amax = block_max(amax);
  const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-12f);
  const float rs = __frcp_rn(s);
  if (threadIdx.x == 0) scale[r] = s;
  uint2* qr = reinterpret_cast<uint2*>(q + r * ldq);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int vi = threadIdx.x + THREADS * i;
    if (vi >= nvec) continue;
    const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
    uint32_t packed[2] = {0u, 0u};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float f = __uint_as_float((e & 1) ? (w[e >> 1] & 0xFFFF0000u) : (w[e >> 1] << 16));
      const float c = fminf(fmaxf(rint_quotient(f, s, rs), -127.f), 127.f);
      packed[e >> 2] |= (uint32_t)(static_cast<int>(c) & 0xFF) << (8 * (e & 3));
    }
    qr[vi] = make_uint2(packed[0], packed[1]);
  }
}

// Per-row int8 with the row amax already known (accumulated by the producing GEMM's
// epilogue): one streaming pass, block (row, 256-vector chunk), 8 codes per thread.
__global__ void __launch_bounds__(256) int8_rows_amax_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                              int K, const float* __restrict__ amax,
                                                              int8_t* __restrict__ q, long long ldq,
                                                              float* __restrict__ scale) {
  const long long r = blockIdx.x;
  const int vi = blockIdx.y * 256 + threadIdx.x;
  const float s = fmaxf(__fdiv_rn(amax[r], 127.0f), 1e-12f);
  const float rs = __frcp_rn(s);
  if (vi == 0) scale[r] = s;
  if (vi >= (K >> 3)) return;
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(x + r * ldx) + vi);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t packed[2] = {0u, 0u};
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float f = __uint_as_float((e & 1) ? (w[e >> 1] & 0xFFFF0000u) : (w[e >> 1] << 16));
    const float c = fminf(fmaxf(rint_quotient(f, s, rs), -127.f), 127.f);
    packed[e >> 2] |= (uint32_t)(static_cast<int>(c) & 0xFF) << (8 * (e & 3));
  }
  reinterpret_cast<uint2*>(q + r * ldq)[vi] = make_uint2(packed[0], packed[1]);
}

// Per-tensor amax and e4m3 cast: CTAs stride over rows, threads over a row's columns (no
// per-element index division); VEC: aligned bf16 rows read 8 at a time with 16-byte loads.
// The per-element arithmetic is the same in every variant.
template <typename T, bool VEC>
__global__ void amax_kernel(const T* __restrict__ x, long long ldx, int rows, int K, float* __restrict__ amax) {
  float m = 0.f;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* row = x + (long long)r * ldx;
    if constexpr (VEC) {
      const uint4* rv = reinterpret_cast<const uint4*>(row);
      for (int vi = threadIdx.x; vi < (K >> 3); vi += blockDim.x) {
        const uint4 v = __ldg(rv + vi);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e)
          m = fmaxf(m, fmaxf(fabsf(__uint_as_float(w[e] << 16)), fabsf(__uint_as_float(w[e] & 0xFFFF0000u))));
      }
    } else {
      for (int c = threadIdx.x; c < K; c += blockDim.x) m = fmaxf(m, fabsf(to_f<T>(row[c])));
    }
  }
  m = block_max(m);
  if (threadIdx.x == 0) atomicMax(reinterpret_cast<int*>(amax), __float_as_int(m));
}

__device__ __forceinline__ uint32_t e4m3_code(float f, float s) {
  float v = __fdiv_rn(f, s);
  v = fminf(fmaxf(v, -448.f), 448.f);
  return (uint32_t)__nv_fp8_e4m3(v).__x;
}

template <typename T, bool VEC>
__global__ void fp8_cast_kernel(const T* __restrict__ x, long long ldx, int rows, int K, const float* __restrict__ amax,
                                __nv_fp8_e4m3* __restrict__ q, long long ldq, float* __restrict__ scale_out) {
  const float s = fmaxf(__fdiv_rn(*amax, 448.0f), 1e-12f);
  if (blockIdx.x == 0 && threadIdx.x == 0 && scale_out) *scale_out = s;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* row = x + (long long)r * ldx;
    __nv_fp8_e4m3* qr = q + (long long)r * ldq;
    if constexpr (VEC) {
      const uint4* rv = reinterpret_cast<const uint4*>(row);
      for (int vi = threadIdx.x; vi < (K >> 3); vi += blockDim.x) {
        const uint4 v = __ldg(rv + vi);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t packed[2] = {0u, 0u};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float f = __uint_as_float((e & 1) ? (w[e >> 1] & 0xFFFF0000u) : (w[e >> 1] << 16));
          packed[e >> 2] |= e4m3_code(f, s) << (8 * (e & 3));
        }
        reinterpret_cast<uint2*>(qr)[vi] = make_uint2(packed[0], packed[1]);
      }
    } else {
      for (int c = threadIdx.x; c < K; c += blockDim.x) qr[c].__x = (__nv_fp8_storage_t)e4m3_code(to_f<T>(row[c]), s);
    }
  }
}

// Grid of the two per-tensor passes: CTAs stride over rows, at most 4 per SM.
inline int tensor_pass_blocks(int rows) { return std::max(1, std::min(rows, 4 * vdn::sm_count())); }

inline bool bf16_rows_vec(int src_kind, const void* x, long long ldx, int K, const void* q, long long ldq) {
  return src_kind == 0 && K % 8 == 0 && vdn::aligned16(x) && ldx % 8 == 0 &&
         (q == nullptr || ((reinterpret_cast<uintptr_t>(q) & 7) == 0 && ldq % 8 == 0));
}

inline void launch_amax(int src_kind, const void* x, long long ldx, int rows, int K, float* amax, cudaStream_t s) {
  const int blocks = tensor_pass_blocks(rows);
  if (bf16_rows_vec(src_kind, x, ldx, K, nullptr, 0))
    amax_kernel<__nv_bfloat16, true><<<blocks, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(x), ldx, rows, K,
                                                            amax);
  else if (src_kind == 0)
    amax_kernel<__nv_bfloat16, false><<<blocks, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(x), ldx, rows, K,
                                                             amax);
  else
    amax_kernel<float, false><<<blocks, 256, 0, s>>>(reinterpret_cast<const float*>(x), ldx, rows, K, amax);
  vdn::count_launch();
}

inline void launch_fp8_cast(int src_kind, const void* x, long long ldx, int rows, int K, const float* amax, void* q,
                            long long ldq, float* scale_out, cudaStream_t s) {
  const int blocks = tensor_pass_blocks(rows);
  auto qb = reinterpret_cast<__nv_fp8_e4m3*>(q);
  if (bf16_rows_vec(src_kind, x, ldx, K, q, ldq))
    fp8_cast_kernel<__nv_bfloat16, true><<<blocks, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(x), ldx, rows,
                                                                K, amax, qb, ldq, scale_out);
  else if (src_kind == 0)
    fp8_cast_kernel<__nv_bfloat16, false><<<blocks, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(x), ldx,
                                                                 rows, K, amax, qb, ldq, scale_out);
  else
    fp8_cast_kernel<float, false><<<blocks, 256, 0, s>>>(reinterpret_cast<const float*>(x), ldx, rows, K, amax, qb,
                                                         ldq, scale_out);
  vdn::count_launch();
}

// ConvRot rows: each 256-wide group of a row is rotated by H = R/16, R the fourth Kronecker
// power of the order-4 regular Hadamard matrix J - 2I (symmetric, H H = I), then the rotated
// row is quantised per row like int8_rows_vec_kernel.  Rotating both the activation rows and
// the weight rows leaves x W^T unchanged, and spreads a channel outlier over its group.
//
// A warp owns one group at a time, a lane 8 consecutive elements (index i = 8 lane + e).  The
// group index has four base-4 digits, d0 = e & 3, d1 = (e >> 2) | (lane & 1) << 1,
// d2 = (lane >> 1) & 3, d3 = lane >> 3; R applies J - 2I along each digit in the order
// d0, d1, d2, d3: y = S - 2 x with S = (x[d=0] + x[d=1]) + (x[d=2] + x[d=3]).  Every lane of a
// quadruple forms S from the same two pair sums (IEEE addition commutes exactly), so the
// result is one fixed fp32 sequence that a CPU restatement reproduces bit for bit.
// Block: WARPS warps, a row per CTA; warp w rotates groups w, w + WARPS, ... (G at most).
template <int G, int WARPS>
__global__ void __launch_bounds__(WARPS * 32) int8_rows_convrot_kernel(const __nv_bfloat16* __restrict__ x,
                                                                      long long ldx, int K, int8_t* __restrict__ q,
                                                                      long long ldq, float* __restrict__ scale) {
  const long long r = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int groups = K >> 8;
  const __nv_bfloat16* row = x + r * ldx;
  float v[G][8];
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const int g = warp + WARPS * j;
    if (g >= groups) {  // warp-uniform
#pragma unroll
      for (int e = 0; e < 8; ++e) v[j][e] = 0.f;
      continue;
    }
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(row + ((long long)g << 8)) + lane);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int e = 0; e < 8; ++e) v[j][e] = __uint_as_float((e & 1) ? (w[e >> 1] & 0xFFFF0000u) : (w[e >> 1] << 16));
    // d0: four consecutive elements in registers
#pragma unroll
    for (int b = 0; b < 8; b += 4) {
      const float s = (v[j][b] + v[j][b + 1]) + (v[j][b + 2] + v[j][b + 3]);
#pragma unroll
      for (int t = 0; t < 4; ++t) v[j][b + t] = s - 2.f * v[j][b + t];
    }
    // d1: element bit 2 in registers, lane bit 0 across the pair of lanes
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float p = v[j][t] + v[j][t + 4];
      const float s = p + __shfl_xor_sync(0xffffffffu, p, 1);
      v[j][t] = s - 2.f * v[j][t];
      v[j][t + 4] = s - 2.f * v[j][t + 4];
    }
    // d2: lane bits 1-2; d3: lane bits 3-4
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float p = v[j][e] + __shfl_xor_sync(0xffffffffu, v[j][e], 2);
      const float s = p + __shfl_xor_sync(0xffffffffu, p, 4);
      v[j][e] = s - 2.f * v[j][e];
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float p = v[j][e] + __shfl_xor_sync(0xffffffffu, v[j][e], 8);
      const float s = p + __shfl_xor_sync(0xffffffffu, p, 16);
      v[j][e] = (s - 2.f * v[j][e]) * 0.0625f;
      amax = fmaxf(amax, fabsf(v[j][e]));
    }
  }
  amax = block_max(amax);
  const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-12f);
  const float rs = __frcp_rn(s);
  if (threadIdx.x == 0) scale[r] = s;
  int8_t* qr = q + r * ldq;
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const int g = warp + WARPS * j;
    if (g >= groups) continue;
    uint32_t packed[2] = {0u, 0u};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float c = fminf(fmaxf(rint_quotient(v[j][e], s, rs), -127.f), 127.f);
      packed[e >> 2] |= (uint32_t)(static_cast<int>(c) & 0xFF) << (8 * (e & 3));
    }
    reinterpret_cast<uint2*>(qr + ((long long)g << 8))[lane] = make_uint2(packed[0], packed[1]);
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
  const bool vec = src_kind == 0 && K % 8 == 0 && K <= 8 * 1024 * 4 && vdn::aligned16(x) && (ldx * 2) % 16 == 0 &&
                   (reinterpret_cast<uintptr_t>(q) & 7) == 0 && ldq % 8 == 0;
  if (vec) {
    const int nvec = K / 8;
    const auto xb = reinterpret_cast<const __nv_bfloat16*>(x);
    const auto qb = reinterpret_cast<int8_t*>(q);
    if (nvec <= 256 * 2)
      vdn::quant::int8_rows_vec_kernel<2, 256><<<rows, 256, 0, s>>>(xb, ldx, K, qb, ldq, scale);
    else if (nvec <= 256 * 4)
      vdn::quant::int8_rows_vec_kernel<4, 256><<<rows, 256, 0, s>>>(xb, ldx, K, qb, ldq, scale);
    else
      vdn::quant::int8_rows_vec_kernel<4, 1024><<<rows, 1024, 0, s>>>(xb, ldx, K, qb, ldq, scale);
  } else if (src_kind == 0)
    vdn::quant::int8_rows_kernel<__nv_bfloat16><<<rows, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(x), ldx, K,
                                                                      reinterpret_cast<int8_t*>(q), ldq, scale);
  else
    vdn::quant::int8_rows_kernel<float><<<rows, 256, 0, s>>>(reinterpret_cast<const float*>(x), ldx, K,
                                                              reinterpret_cast<int8_t*>(q), ldq, scale);
  vdn::count_launch();
  return vdn::launch_status();
}

// Per-row symmetric int8 of bf16 rows whose max |x| per row is already in amax [rows] (the
// same codes and scales as vdn_quant_int8_rows).  K % 8 == 0, 16-byte aligned x rows, 8-byte
// aligned q rows.
int vdn_quant_int8_rows_amax(const void* x, long long ldx, int rows, int K, const float* amax, void* q,
                             long long ldq, float* scale, void* stream) {
  if (!x || !q || !scale || !amax || rows < 0 || K <= 0) return vdn::kBadArgument;
  if (K % 8) return vdn::kUnsupported;
  if (!vdn::aligned16(x) || (ldx * 2) % 16 || (reinterpret_cast<uintptr_t>(q) & 7) || ldq % 8)
    return vdn::kMisaligned;
  if (rows == 0) return vdn::kOk;
  const dim3 grid((unsigned)rows, (unsigned)((K / 8 + 255) / 256));
  vdn::quant::int8_rows_amax_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), ldx, K, amax, reinterpret_cast<int8_t*>(q), ldq, scale);
  vdn::count_launch();
  return vdn::launch_status();
}

// ConvRot int8 rows (group 256): rotate each 256-wide group of a bf16 row, then per-row
// symmetric int8 as vdn_quant_int8_rows.  K % 256 == 0, K <= 32768; x rows 16-byte aligned,
// q rows 8-byte aligned.
int vdn_quant_int8_rows_convrot(const void* x, long long ldx, int rows, int K, int group, void* q, long long ldq,
                                float* scale, void* stream) {
  if (!x || !q || !scale || rows < 0 || K <= 0) return vdn::kBadArgument;
  if (group != 256 || K % 256 || K > 32768) return vdn::kUnsupported;
  if (!vdn::aligned16(x) || (ldx * 2) % 16 || (reinterpret_cast<uintptr_t>(q) & 7) || ldq % 8)
    return vdn::kMisaligned;
  if (rows == 0) return vdn::kOk;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  const auto xb = reinterpret_cast<const __nv_bfloat16*>(x);
  const auto qb = reinterpret_cast<int8_t*>(q);
  const int groups = K / 256;
  if (groups <= 8)
    vdn::quant::int8_rows_convrot_kernel<1, 8><<<rows, 256, 0, s>>>(xb, ldx, K, qb, ldq, scale);
  else if (groups <= 16)
    vdn::quant::int8_rows_convrot_kernel<2, 8><<<rows, 256, 0, s>>>(xb, ldx, K, qb, ldq, scale);
  else if (groups <= 24)
    vdn::quant::int8_rows_convrot_kernel<3, 8><<<rows, 256, 0, s>>>(xb, ldx, K, qb, ldq, scale);
  else if (groups <= 32)
    vdn::quant::int8_rows_convrot_kernel<4, 8><<<rows, 256, 0, s>>>(xb, ldx, K, qb, ldq, scale);
  else if (groups <= 64)
    vdn::quant::int8_rows_convrot_kernel<2, 32><<<rows, 1024, 0, s>>>(xb, ldx, K, qb, ldq, scale);
  else
    vdn::quant::int8_rows_convrot_kernel<4, 32><<<rows, 1024, 0, s>>>(xb, ldx, K, qb, ldq, scale);
  vdn::count_launch();
  return vdn::launch_status();
}

// Per-tensor e4m3.  work: one fp32 device scalar (zeroed here) that receives the amax;
// scale_out: the fp32 dequantisation scale.  src_kind 0 = bf16, 1 = fp32.
int vdn_quant_fp8_tensor(int src_kind, const void* x, long long ldx, int rows, int K, void* q, long long ldq,
                         float* work, float* scale_out, void* stream) {
  if (!x || !q || !work || !scale_out || rows < 0 || K <= 0) return vdn::kBadArgument;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  cudaMemsetAsync(work, 0, sizeof(float), s);
  if ((long long)rows * K > 0) {
    vdn::quant::launch_amax(src_kind, x, ldx, rows, K, work, s);
    vdn::quant::launch_fp8_cast(src_kind, x, ldx, rows, K, work, q, ldq, scale_out, s);
  }
  return vdn::launch_status();
}

// The two halves of vdn_quant_fp8_tensor, for callers that combine the amax of several
// devices in between (an all-reduce MAX of `amax` across the ranks of a row-split
// projection): vdn_fp8_amax clears and fills `amax`; vdn_fp8_cast quantises with it.
int vdn_fp8_amax(int src_kind, const void* x, long long ldx, int rows, int K, float* amax, void* stream) {
  if (!x || !amax || rows < 0 || K <= 0) return vdn::kBadArgument;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  cudaMemsetAsync(amax, 0, sizeof(float), s);
  if ((long long)rows * K > 0) vdn::quant::launch_amax(src_kind, x, ldx, rows, K, amax, s);
  return vdn::launch_status();
}

int vdn_fp8_cast(int src_kind, const void* x, long long ldx, int rows, int K, const float* amax, void* q,
                 long long ldq, float* scale_out, void* stream) {
  if (!x || !q || !amax || rows < 0 || K <= 0) return vdn::kBadArgument;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if ((long long)rows * K > 0) vdn::quant::launch_fp8_cast(src_kind, x, ldx, rows, K, amax, q, ldq, scale_out, s);
  return vdn::launch_status();
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// FP8 projection that allocates nothing.
//
// Some callers cannot allocate device memory while they run this projection: code that
// executes inside a memory pool or arena it does not own, embedded hosts that hand the
// library a fixed device budget at start-up, and callers on paths where an allocation
// would synchronise or fail (for example while the caching allocator is exhausted).  For
// them the quantised activations, the amax and the activation scale of the FP8 projection
// live in one file-scope device array instead of buffers the caller provides.
//
// Limits and behaviour:
//   * the array holds at most kNoAllocMaxElems (16 Mi) quantised activation elements, so
//     rows * K must not exceed 16,777,216; larger calls return kTooLarge and do nothing;
//   * every GPU that loads this library keeps the array (about 16 MiB) until the process
//     exits;
//   * the first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (with that device current) and caches it; make that first call
//     before any stream capture;
//   * all calls share the array and it keeps the previous call's contents: the amax word is
//     cleared on the stream at the start of every call, and two calls that overlap on the
//     GPU (different streams, no ordering between them) race on the array.
// ---------------------------------------------------------------------------------------
namespace vdn {
namespace quant {

constexpr long long kNoAllocMaxElems = 16ll * 1024 * 1024;
constexpr long long kNoAllocHeader = 256;  // amax at byte 0, scale at byte 128
static __device__ __align__(256) unsigned char g_fp8_noalloc_scratch[kNoAllocHeader + kNoAllocMaxElems];

// The array's device address on the current device, looked up once per device (atomic
// slots: entry points may be called from several host threads; a lost race looks the same
// address up twice).
static unsigned char* noalloc_scratch_on_current_device() {
  static std::atomic<unsigned char*> addr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  unsigned char* cached = addr[dev].load(std::memory_order_acquire);
  if (!cached) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_fp8_noalloc_scratch) != cudaSuccess) return nullptr;
    cached = static_cast<unsigned char*>(p);
    addr[dev].store(cached, std::memory_order_release);
  }
  return cached;
}

}  // namespace quant
}  // namespace vdn

extern "C" int vdn_gemm(int kind, const void* A, long long lda, const void* A2, long long lda2, long long k_split,
                        const void* B, long long ldb, void* C, long long ldc, int out_kind, int M, int N, int K,
                        float alpha, const float* dev_scale0, const float* dev_scale1, const float* row_scale,
                        const float* col_scale, const float* col_bias, int act, const void* addend,
                        long long ld_add, int* dev_err, void* stream);

extern "C" {

// out[M, N] (bf16) = x[M, K] (bf16) * W^T with x quantised to e4m3 per tensor inside the
// library's own scratch array (see the block comment above), W [N, K] e4m3 with its
// per-tensor scale w_scale (device fp32).  Same result as vdn_quant_fp8_tensor followed by
// vdn_gemm(kind = 1).  Returns kTooLarge when M * K exceeds 16 Mi elements, kBadArgument
// when a row pitch is shorter than its row (ldx or ldw < K, ldo < N).
int vdn_fp8_linear_noalloc(const void* x, long long ldx, int M, int K, const void* w_fp8, long long ldw, int N,
                           const float* w_scale, void* out, long long ldo, int* dev_err, void* stream) {
  if (!x || !w_fp8 || !w_scale || !out || M <= 0 || N <= 0 || K <= 0) return vdn::kBadArgument;
  if (ldx < K || ldw < K || ldo < N) return vdn::kBadArgument;  // rows must not overlap
  if ((long long)M * K > vdn::quant::kNoAllocMaxElems) return vdn::kTooLarge;
  if (K % 16) return vdn::kMisaligned;  // quantised rows are packed at pitch K bytes
  unsigned char* base = vdn::quant::noalloc_scratch_on_current_device();
  if (!base) return vdn::kLaunchFailed;
  float* amax = reinterpret_cast<float*>(base);
  float* scale = reinterpret_cast<float*>(base + 128);
  __nv_fp8_e4m3* q = reinterpret_cast<__nv_fp8_e4m3*>(base + vdn::quant::kNoAllocHeader);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(amax, 0, sizeof(float), s) != cudaSuccess) return vdn::kLaunchFailed;
  vdn::quant::launch_amax(0, x, ldx, M, K, amax, s);
  vdn::quant::launch_fp8_cast(0, x, ldx, M, K, amax, q, K, scale, s);
  const int rc = vdn::launch_status();
  if (rc) return rc;
  return vdn_gemm(1, q, K, nullptr, 0, 0, w_fp8, ldw, out, ldo, 0, M, N, K, 1.0f, scale, w_scale, nullptr, nullptr,
                  nullptr, 0, nullptr, 0, dev_err, stream);
}

}  // extern "C"
