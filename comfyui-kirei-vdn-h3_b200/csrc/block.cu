// Pointwise stretches of the DiT block around the hybrid attention (block_kernels.py:85-93).
//
// The pre-norm of both residual branches, RMSNorm(x) * (1 + scale[g]) + shift[g] with g the
// modulation row of each token, reads x from HBM once: a CTA owns a row held in registers,
// reduces its sum of squares and writes the modulated row as bf16 and/or as per-token int8
// codes with their scale (the quantiser of the INT8 projections, applied to the row it just
// produced).  Rows wider than 32,768 fall back to a warp per row with streaming passes.
// Roundings follow the reference's bf16 tensors: the RMSNorm output, 1 + scale, the product
// and the sum are each rounded to bf16.
// The gated residual x + gate[g] * y is fused into the epilogue of the GEMM that makes y
// (gemm.cu), so no other pass over the residual stream exists.
#include "host_common.h"
#include "sm100.cuh"

namespace vdn {
namespace block {

constexpr int kRowsPerBlock = 8;  // one warp per row

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// Modulated RMSNorm of 8 consecutive columns (one 16-byte vector `vi`) of a row.
__device__ __forceinline__ void modulate8(uint4 xv, uint4 s4, uint4 h4, const float* __restrict__ w, int vi,
                                          float rstd, float (&y)[8]) {
  const float4 w0 = __ldg(reinterpret_cast<const float4*>(w) + 2 * vi);
  const float4 w1 = __ldg(reinterpret_cast<const float4*>(w) + 2 * vi + 1);
  const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  const uint32_t xp[4] = {xv.x, xv.y, xv.z, xv.w};
  const uint32_t sp[4] = {s4.x, s4.y, s4.z, s4.w};
  const uint32_t hp[4] = {h4.x, h4.y, h4.z, h4.w};
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const bool hi = e & 1;
    const float xe = hi ? bf_hi(xp[e >> 1]) : bf_lo(xp[e >> 1]);
    const float se = hi ? bf_hi(sp[e >> 1]) : bf_lo(sp[e >> 1]);
    const float he = hi ? bf_hi(hp[e >> 1]) : bf_lo(hp[e >> 1]);
    const float n = bf16_round(xe * rstd * wv[e]);
    y[e] = bf16_round(bf16_round(n * bf16_round(1.0f + se)) + he);
  }
}

// One warp per row, streaming passes over the row's 16-byte vectors: sum of squares; the
// modulated row (bf16 out, amax); the int8 codes.
__global__ void __launch_bounds__(256) adaln_rmsnorm_kernel(
    const __nv_bfloat16* __restrict__ x, long long ldx, int rows, int hidden, const float* __restrict__ w, float eps,
    const __nv_bfloat16* __restrict__ scale_tab, const __nv_bfloat16* __restrict__ shift_tab, long long ld_tab,
    const int* __restrict__ row_group, __nv_bfloat16* __restrict__ out, long long ldo, int8_t* __restrict__ q,
    long long ldq, float* __restrict__ q_scale) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * kRowsPerBlock + warp;
  if (row >= rows) return;
  const int nvec = hidden >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx);
  float ss = 0.f;
#pragma unroll 4
  for (int vi = lane; vi < nvec; vi += 32) {
    const uint4 v = __ldg(xr + vi);
    const uint32_t p[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) ss += bf_lo(p[e]) * bf_lo(p[e]) + bf_hi(p[e]) * bf_hi(p[e]);
  }
  const float rstd = rsqrtf(warp_sum(ss) / (float)hidden + eps);
  const long long g = row_group ? row_group[row] : 0;
  const uint4* sc = scale_tab ? reinterpret_cast<const uint4*>(scale_tab + g * ld_tab) : nullptr;
  const uint4* sh = shift_tab ? reinterpret_cast<const uint4*>(shift_tab + g * ld_tab) : nullptr;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  float amax = 0.f;
#pragma unroll 2
  for (int vi = lane; vi < nvec; vi += 32) {
    float y[8];
    modulate8(__ldg(xr + vi), sc ? __ldg(sc + vi) : zero, sh ? __ldg(sh + vi) : zero, w, vi, rstd, y);
#pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(y[e]));
    if (out)
      reinterpret_cast<uint4*>(out + row * ldo)[vi] =
          make_uint4(pack_bf16(y[0], y[1]), pack_bf16(y[2], y[3]), pack_bf16(y[4], y[5]), pack_bf16(y[6], y[7]));
  }
  if (!q) return;
  // per-token int8 (quant.cu's rule): scale = max(amax / 127, 1e-12), q = rne(y / scale)
  const float s = fmaxf(__fdiv_rn(warp_max(amax), 127.0f), 1e-12f);
  if (lane == 0) q_scale[row] = s;
#pragma unroll 2
  for (int vi = lane; vi < nvec; vi += 32) {
    float y[8];
    modulate8(__ldg(xr + vi), sc ? __ldg(sc + vi) : zero, sh ? __ldg(sh + vi) : zero, w, vi, rstd, y);
    uint32_t packed[2] = {0u, 0u};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float c = fminf(fmaxf(rintf(__fdiv_rn(y[e], s)), -127.f), 127.f);
      packed[e >> 2] |= (uint32_t)(static_cast<int>(c) & 0xFF) << (8 * (e & 3));
    }
    reinterpret_cast<uint2*>(q + row * ldq)[vi] = make_uint2(packed[0], packed[1]);
  }
}

// Block-wide sum / max through shared memory (every thread gets the result).
template <bool kMax>
__device__ __forceinline__ float block_reduce(float v, float* red) {
  v = kMax ? warp_max(v) : warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = l < (int)(blockDim.x >> 5) ? red[l] : 0.f;
    v = kMax ? warp_max(v) : warp_sum(v);
    if (l == 0) red[32] = v;
  }
  __syncthreads();
  const float r = red[32];
  __syncthreads();
  return r;
}

// One CTA per row with the row in registers (NV 16-byte vectors per thread, hidden <= 8 *
// THREADS * NV): x is read once, the modulated row is kept packed for the int8 codes.
template <int NV, int THREADS>
__global__ void __launch_bounds__(THREADS) adaln_rmsnorm_row_kernel(
    const __nv_bfloat16* __restrict__ x, long long ldx, int hidden, const float* __restrict__ w, float eps,
    const __nv_bfloat16* __restrict__ scale_tab, const __nv_bfloat16* __restrict__ shift_tab, long long ld_tab,
    const int* __restrict__ row_group, __nv_bfloat16* __restrict__ out, long long ldo, int8_t* __restrict__ q,
    long long ldq, float* __restrict__ q_scale) {
  __shared__ float red[33];
  const long long row = blockIdx.x;
  const int nvec = hidden >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx);
  uint4 v[NV];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int vi = threadIdx.x + THREADS * i;
    v[i] = vi < nvec ? __ldg(xr + vi) : make_uint4(0, 0, 0, 0);
    const uint32_t p[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) ss += bf_lo(p[e]) * bf_lo(p[e]) + bf_hi(p[e]) * bf_hi(p[e]);
  }
  const float rstd = rsqrtf(block_reduce<false>(ss, red) / (float)hidden + eps);
  const long long g = row_group ? row_group[row] : 0;
  const uint4* sc = scale_tab ? reinterpret_cast<const uint4*>(scale_tab + g * ld_tab) : nullptr;
  const uint4* sh = shift_tab ? reinterpret_cast<const uint4*>(shift_tab + g * ld_tab) : nullptr;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int vi = threadIdx.x + THREADS * i;
    if (vi >= nvec) continue;
    float y[8];
    modulate8(v[i], sc ? __ldg(sc + vi) : zero, sh ? __ldg(sh + vi) : zero, w, vi, rstd, y);
#pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(y[e]));
    v[i] = make_uint4(pack_bf16(y[0], y[1]), pack_bf16(y[2], y[3]), pack_bf16(y[4], y[5]), pack_bf16(y[6], y[7]));
    if (out) reinterpret_cast<uint4*>(out + row * ldo)[vi] = v[i];
  }
  if (!q) return;
  const float s = fmaxf(__fdiv_rn(block_reduce<true>(amax, red), 127.0f), 1e-12f);
  if (threadIdx.x == 0) q_scale[row] = s;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int vi = threadIdx.x + THREADS * i;
    if (vi >= nvec) continue;
    const uint32_t yp[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
    uint32_t packed[2] = {0u, 0u};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float yv = (e & 1) ? bf_hi(yp[e >> 1]) : bf_lo(yp[e >> 1]);
      const float c = fminf(fmaxf(rintf(__fdiv_rn(yv, s)), -127.f), 127.f);
      packed[e >> 2] |= (uint32_t)(static_cast<int>(c) & 0xFF) << (8 * (e & 3));
    }
    reinterpret_cast<uint2*>(q + row * ldq)[vi] = make_uint2(packed[0], packed[1]);
  }
}

// ---------------------------------------------------------------------------------
// Rotary position embedding on the normalised q / k heads, split-half pairing: for each
// head slot and j < rot/2 the pair (x[j], x[j + rot/2]) becomes f[j] (x[j], x[j + rot/2])^T
// with f[j] the token's 2 x 2 matrix in ComfyUI's freqs layout ([..., rot/2, 2, 2] =
// [[cos, -sin], [sin, cos]]); features >= rot pass through.  In place, fp32 arithmetic, one
// bf16 rounding.
//
// Vector path (rot % 16 == 0): one warp per token row, 8 rows per CTA; lane l takes the
// 16-byte groups v = l, l + 32, ... of the row's slots x G groups of 8 pairs (G = rot / 16).
// When G divides 32 a lane's pair group is the same for every v, so its 8 matrices are
// read once per row into registers (L1 serves the lanes sharing them).
template <bool kFixedGroup>
__global__ void __launch_bounds__(256) rope_split_half_vec_kernel(__nv_bfloat16* __restrict__ qk, long long ld,
                                                                  int rows, int slots, int D, int half,
                                                                  const float* __restrict__ freqs, long long ld_freqs) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * 8 + warp;
  if (row >= rows) return;
  const int G = half / 8;
  const float4* fr = reinterpret_cast<const float4*>(freqs + row * ld_freqs);
  __nv_bfloat16* base = qk + row * ld;
  float4 f[8];
  if (kFixedGroup) {
    const int g = lane % G;
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = __ldg(fr + g * 8 + i);
  }
  const int n = slots * G;
#pragma unroll 2
  for (int v = lane; v < n; v += 32) {
    const int slot = v / G, g = v - slot * G;
    if (!kFixedGroup) {
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = __ldg(fr + g * 8 + i);
    }
    __nv_bfloat16* p1 = base + (long long)slot * D + g * 8;
    __nv_bfloat16* p2 = p1 + half;
    const uint4 a = *reinterpret_cast<const uint4*>(p1);
    const uint4 b = *reinterpret_cast<const uint4*>(p2);
    const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&b);
    uint4 oa, ob;
    uint32_t* aw = reinterpret_cast<uint32_t*>(&oa);
    uint32_t* bw = reinterpret_cast<uint32_t*>(&ob);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x1 = __bfloat1622float2(a2[i]), x2 = __bfloat1622float2(b2[i]);
      const float4 f0 = f[2 * i], f1 = f[2 * i + 1];
      aw[i] = pack_bf16(fmaf(f0.y, x2.x, f0.x * x1.x), fmaf(f1.y, x2.y, f1.x * x1.y));
      bw[i] = pack_bf16(fmaf(f0.w, x2.x, f0.z * x1.x), fmaf(f1.w, x2.y, f1.z * x1.y));
    }
    *reinterpret_cast<uint4*>(p1) = oa;
    *reinterpret_cast<uint4*>(p2) = ob;
  }
}

// Scalar path (any even rot): one CTA per token row, the row's matrices staged in shared
// memory, one pair per thread step.
__global__ void __launch_bounds__(256) rope_split_half_kernel(__nv_bfloat16* __restrict__ qk, long long ld, int slots,
                                                              int D, int half, const float* __restrict__ freqs,
                                                              long long ld_freqs) {
  extern __shared__ float fm[];  // [half][2][2]
  const long long row = blockIdx.x;
  const float* fr = freqs + row * ld_freqs;
  for (int e = threadIdx.x; e < half * 4; e += blockDim.x) fm[e] = fr[e];
  __syncthreads();
  __nv_bfloat16* base = qk + row * ld;
  for (int v = threadIdx.x; v < slots * half; v += blockDim.x) {
    const int slot = v / half, j = v - slot * half;
    __nv_bfloat16* p1 = base + (long long)slot * D + j;
    const float x1 = __bfloat162float(p1[0]), x2 = __bfloat162float(p1[half]);
    p1[0] = __float2bfloat16_rn(fmaf(fm[4 * j + 1], x2, fm[4 * j] * x1));
    p1[half] = __float2bfloat16_rn(fmaf(fm[4 * j + 3], x2, fm[4 * j + 2] * x1));
  }
}

}  // namespace block
}  // namespace vdn

extern "C" {

// out / q[r] = RMSNorm(x[r]) * norm_w * (1 + scale_tab[g]) + shift_tab[g], g = row_group[r]
// (block_kernels.py:85-89).  x [rows, ldx] bf16; norm_w [hidden] fp32; scale_tab / shift_tab
// [groups, ld_tab] bf16 (either may be NULL: scale 0 / shift 0); row_group [rows] int32 (NULL:
// every row uses group 0).  Writes out [rows, ldo] bf16 and/or q [rows, ldq] int8 with
// q_scale [rows] fp32 (per-token int8 of the modulated row).  hidden % 8 == 0; 16-byte aligned
// rows (8-byte for q).
int vdn_adaln_rmsnorm(const void* x, long long ldx, int rows, int hidden, const float* norm_w, float eps,
                      const void* scale_tab, const void* shift_tab, long long ld_tab, const int* row_group,
                      void* out, long long ldo, void* q, long long ldq, float* q_scale, void* stream) {
  if (!x || !norm_w || (!out && !q) || (q && !q_scale) || rows < 0 || hidden <= 0) return vdn::kBadArgument;
  if (hidden % 8) return vdn::kUnsupported;
  if (!vdn::aligned16(x) || (ldx * 2) % 16 || !vdn::aligned16(norm_w)) return vdn::kMisaligned;
  if (out && (!vdn::aligned16(out) || (ldo * 2) % 16)) return vdn::kMisaligned;
  if (q && ((reinterpret_cast<uintptr_t>(q) & 7) || ldq % 8)) return vdn::kMisaligned;
  if ((scale_tab && !vdn::aligned16(scale_tab)) || (shift_tab && !vdn::aligned16(shift_tab)) ||
      ((scale_tab || shift_tab) && (ld_tab * 2) % 16))
    return vdn::kMisaligned;
  if (rows == 0) return vdn::kOk;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  const int nvec = hidden / 8;
  const auto xb = reinterpret_cast<const __nv_bfloat16*>(x);
  const auto st = reinterpret_cast<const __nv_bfloat16*>(scale_tab);
  const auto ht = reinterpret_cast<const __nv_bfloat16*>(shift_tab);
  const auto ob = reinterpret_cast<__nv_bfloat16*>(out);
  const auto qb = reinterpret_cast<int8_t*>(q);
  if (nvec <= 256 * 2) {
    vdn::block::adaln_rmsnorm_row_kernel<2, 256><<<(unsigned)rows, 256, 0, s>>>(
        xb, ldx, hidden, norm_w, eps, st, ht, ld_tab, row_group, ob, ldo, qb, ldq, q_scale);
    vdn::count_launch();
    return vdn::launch_status();
  }
  if (nvec <= 256 * 4) {
    vdn::block::adaln_rmsnorm_row_kernel<4, 256><<<(unsigned)rows, 256, 0, s>>>(
        xb, ldx, hidden, norm_w, eps, st, ht, ld_tab, row_group, ob, ldo, qb, ldq, q_scale);
    vdn::count_launch();
    return vdn::launch_status();
  }
  if (nvec <= 1024 * 4) {
    vdn::block::adaln_rmsnorm_row_kernel<4, 1024><<<(unsigned)rows, 1024, 0, s>>>(
        xb, ldx, hidden, norm_w, eps, st, ht, ld_tab, row_group, ob, ldo, qb, ldq, q_scale);
    vdn::count_launch();
    return vdn::launch_status();
  }
  // wider rows: one warp per row, streaming passes
  const unsigned blocks = (unsigned)((rows + vdn::block::kRowsPerBlock - 1) / vdn::block::kRowsPerBlock);
  vdn::block::adaln_rmsnorm_kernel<<<blocks, 32 * vdn::block::kRowsPerBlock, 0, s>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), ldx, rows, hidden, norm_w, eps,
      reinterpret_cast<const __nv_bfloat16*>(scale_tab), reinterpret_cast<const __nv_bfloat16*>(shift_tab), ld_tab,
      row_group, reinterpret_cast<__nv_bfloat16*>(out), ldo, reinterpret_cast<int8_t*>(q), ldq, q_scale);
  vdn::count_launch();
  return vdn::launch_status();
}

// RoPE, split-half pairing, in place on `slots` consecutive heads of D bf16 features per
// row (q heads then k heads of the normalised projection): qk [rows, ld] bf16; freqs fp32
// [rows, rot/2, 2, 2] with row stride ld_freqs (0: one set of matrices for every row).
// rot even, 2 <= rot <= D.  Replaces the RoPE half of comfy-kitchen's
// rms_rope_split_half_(q, k, freqs, ..., rot_dim = 2 * freqs.shape[-3]) (hybrid.py:271-292).
int vdn_rope_split_half(void* qk, long long ld, int rows, int slots, int D, int rot, const float* freqs,
                        long long ld_freqs, void* stream) {
  using namespace vdn::block;
  if (!qk || !freqs || rows < 0 || slots <= 0 || D <= 0 || rot < 2 || rot > D || (rot & 1) || ld < (long long)slots * D ||
      ld_freqs < 0)
    return vdn::kBadArgument;
  if (rows == 0) return 0;
  const int half = rot / 2;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  auto* p = reinterpret_cast<__nv_bfloat16*>(qk);
  const bool vec = half % 8 == 0 && D % 8 == 0 && ld % 8 == 0 && vdn::aligned16(qk) && vdn::aligned16(freqs) &&
                   ld_freqs % 4 == 0;
  if (vec) {
    const unsigned grid = (unsigned)((rows + 7) / 8);
    if (32 % (half / 8) == 0)
      rope_split_half_vec_kernel<true><<<grid, 256, 0, s>>>(p, ld, rows, slots, D, half, freqs, ld_freqs);
    else
      rope_split_half_vec_kernel<false><<<grid, 256, 0, s>>>(p, ld, rows, slots, D, half, freqs, ld_freqs);
  } else {
    rope_split_half_kernel<<<rows, 256, (size_t)half * 4 * sizeof(float), s>>>(p, ld, slots, D, half, freqs,
                                                                              ld_freqs);
  }
  vdn::count_launch();
  return vdn::launch_status();
}

}  // extern "C"
