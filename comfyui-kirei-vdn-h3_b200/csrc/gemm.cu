// Persistent, warp-specialised tcgen05 GEMM for the projections of the VDN-H3 block:
//
//     C[M, N] = epilogue( A[M, K] * B[N, K]^T )        (both operands K-major)
//
// B200 design:
//   * one CTA per SM, static persistent tile loop over 128 x 256 output tiles, grouped
//     along M so a 16-row-tile band of A stays L2-resident while B streams;
//   * warp 0 issues TMA loads (128-byte swizzle) into a 4-stage shared-memory ring;
//   * warp 1 issues tcgen05.mma (M=128, N=256) into one of two TMEM accumulators
//     (2 x 256 fp32 columns), so the epilogue of tile i overlaps the main loop of i+1;
//   * warps 2..9 drain TMEM (tcgen05.ld 32x32b) and apply the fused epilogue: two warps per
//     TMEM lane quarter, each taking half of the tile's columns, so the epilogue (which
//     otherwise sets a per-tile floor of ~38 us) keeps up with the main loop.
// Kinds: 0 = bf16 (kind::f16), 1 = fp8 e4m3 (kind::f8f6f4), 2 = int8 (kind::i8, s32).
//
// Epilogue modes cover every projection of the block:
//   * plain bf16 / fp32 / raw int32 stores, with optional per-row (per-token) and
//     per-column (per-channel) scales, column bias, sigmoid and a bf16 addend;
//   * the QKV epilogue: raw q/k/v in bf16, plus q and k RMS-normalised per head into a
//     second buffer (hybrid.py:271-273 with rope_freqs=None), plus the gate/beta/alpha
//     projection columns (hybrid.py:518-522, branch.py:736, :743-751, :754-758) as fp32;
//   * a K-concatenated A operand (two tensor maps split at k_split), so out_proj and
//     to_out_linear run as one GEMM over [gated softmax | branch readout] (hybrid.py:534-540).
#include "host_common.h"
#include "sm100.cuh"

namespace vdn {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int kStages = 4;
constexpr int kEpiWarps = 8;  // two per TMEM lane quarter, each draining half of the tile's columns
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kStageA = BM * 128;  // bytes: 128 rows x 128 B
constexpr int kStageB = BN * 128;
constexpr int kStageBytes = kStageA + kStageB;
constexpr int kGroupM = 16;

enum OutKind : int { kOutBF16 = 0, kOutF32 = 1, kOutS32 = 2 };

struct Epilogue {
  void* out;
  long long ldo;
  int out_kind;
  int vec_ok;  // 1 when `out` and its row pitch are 16-byte aligned (vector stores allowed)
  int act;  // 0 none, 1 sigmoid, 2 GELU (erf), 3 SwiGLU over paired 128-column blocks
  float alpha;
  const float* row_scale;  // [M]
  const float* col_scale;  // [N]
  const float* dev_scale0; // device scalar multiplied into alpha (per-tensor fp8 scales)
  const float* dev_scale1;
  const float* col_bias;   // [N]
  const __nv_bfloat16* addend;
  long long ld_add;
  // gated residual (block_kernels.py:92-93): out = addend + gate[row_group[row], col] * y, with
  // y and the product rounded to bf16 like the reference's bf16 tensors
  const int* row_group;
  const __nv_bfloat16* group_gate;
  long long ld_group_gate;
  // per-row max |output| (of the bf16-rounded values), accumulated with atomicMax over the
  // row's tiles: the next projection's per-token int8 scale without another pass
  float* row_amax;
  int cs_vec_ok;    // col_scale / col_bias 16-byte aligned: float4 loads
  int cb_vec_ok;
  int add_vec_ok;   // addend rows 16-byte aligned: 8-element vector loads
  int gate_vec_ok;  // gate table rows 16-byte aligned
  // QKV extension
  int norm_cols;  // columns [0, norm_cols) are RMS-normalised per head into norm_out
  int norm_split; // columns < norm_split use norm_w[0:hd], others norm_w[hd:2hd]
  int head_dim;
  float eps;
  __nv_bfloat16* norm_out;
  long long ld_norm;
  const float* norm_w;
  int aux_col0;  // columns >= aux_col0 are written as fp32 to aux_out
  float* aux_out;
  long long ld_aux;
  // branch q features (QKV epilogue): rows [act_row0, act_row0 + act_rows) of the q columns,
  // activated and stored [frame][head][token][head_dim]
  __nv_bfloat16* act_out;
  int act_row0, act_rows, act_tpf, act_heads;
};

// x * sigmoid(x) with the fast reciprocal (the result is rounded to bf16)
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// GELU with the error function (torch.nn.functional.gelu, approximate="none")
__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

enum Act : int { kActNone = 0, kActSigmoid = 1, kActGelu = 2, kActSwiGLU = 3 };

template <int KIND>
struct Traits;
template <>
struct Traits<0> {
  static constexpr int BK = 64, UK = 16;
  static constexpr uint32_t idesc = make_idesc(1, 1, 1, 0, 0, BM, BN);
  __device__ static void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t acc) {
    mma_f16(d, a, b, idesc, acc);
  }
};
template <>
struct Traits<1> {
  static constexpr int BK = 128, UK = 32;
  static constexpr uint32_t idesc = make_idesc(1, 0, 0, 0, 0, BM, BN);
  __device__ static void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t acc) {
    mma_f8(d, a, b, idesc, acc);
  }
};
template <>
struct Traits<2> {
  static constexpr int BK = 128, UK = 32;
  static constexpr uint32_t idesc = make_idesc(2, 1, 1, 0, 0, BM, BN);
  __device__ static void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t acc) {
    mma_i8(d, a, b, idesc, acc);
  }
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& m, int& n) {
  const int per_group = kGroupM * num_n;
  const int g = t / per_group;
  const int first = g * kGroupM;
  const int gsize = min(kGroupM, num_m - first);
  const int local = t - g * per_group;
  m = first + local % gsize;
  n = local / gsize;
}

template <int KIND>
__device__ __forceinline__ float acc_value(uint32_t bits) {
  if constexpr (KIND == 2) {
    return __int2float_rn(static_cast<int>(bits));
  } else {
    return __uint_as_float(bits);
  }
}

// Scaled accumulator value of column `col` (alpha already includes device scalars).
template <int KIND>
__device__ __forceinline__ float scaled(const Epilogue& ep, uint32_t bits, float alpha_rs, int col, int N) {
  float x = acc_value<KIND>(bits) * alpha_rs;
  if (ep.col_scale && col < N) x *= ep.col_scale[col];
  return x;
}

template <int KIND>
__device__ __forceinline__ void store_plain_chunk(const Epilogue& ep, const uint32_t (&r)[32], int row,
                                                  int col0, int M, int N, float alpha) {
  if (row >= M) return;
  if (ep.out_kind == kOutS32) {
    int* dst = reinterpret_cast<int*>(ep.out) + (long long)row * ep.ldo + col0;
    if (ep.vec_ok && col0 + 32 <= N) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<int4*>(dst + j) = make_int4(r[j], r[j + 1], r[j + 2], r[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) dst[j] = static_cast<int>(r[j]);
    }
    return;
  }
  // One branch per optional feature per 32-column chunk (never per element), 16-byte loads
  // of the per-column vectors when the chunk is whole: the epilogue must keep up with a
  // main loop of a few microseconds per tile.
  float v[32];
  const float ars = alpha * (ep.row_scale ? ep.row_scale[row] : 1.0f);
  const bool full = col0 + 32 <= N;
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = acc_value<KIND>(r[j]) * ars;
  if (ep.col_scale) {
    if (full && ep.cs_vec_ok) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 c = __ldg(reinterpret_cast<const float4*>(ep.col_scale + col0 + j));
        v[j] *= c.x, v[j + 1] *= c.y, v[j + 2] *= c.z, v[j + 3] *= c.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) v[j] *= ep.col_scale[col0 + j];
    }
  }
  if (ep.col_bias) {
    if (full && ep.cb_vec_ok) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 c = __ldg(reinterpret_cast<const float4*>(ep.col_bias + col0 + j));
        v[j] += c.x, v[j + 1] += c.y, v[j + 2] += c.z, v[j + 3] += c.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) v[j] += ep.col_bias[col0 + j];
    }
  }
  if (ep.act == kActSigmoid) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = 1.0f / (1.0f + __expf(-v[j]));
  } else if (ep.act == kActGelu) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = gelu_erf(bf16_round(v[j]));
  }
  if (ep.group_gate) {
    const __nv_bfloat16* gate = ep.group_gate + (long long)ep.row_group[row] * ep.ld_group_gate + col0;
    if (ep.gate_vec_ok && full) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        const uint4 p = __ldg(reinterpret_cast<const uint4*>(gate + j));
        const uint32_t w[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float gv = __uint_as_float((e & 1) ? (w[e >> 1] & 0xFFFF0000u) : (w[e >> 1] << 16));
          v[j + e] = bf16_round(bf16_round(v[j + e]) * gv);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) v[j] = bf16_round(bf16_round(v[j]) * __bfloat162float(gate[j]));
    }
  }
  if (ep.addend) {
    const __nv_bfloat16* src = ep.addend + (long long)row * ep.ld_add + col0;
    if (ep.add_vec_ok && full) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        const uint4 p = *reinterpret_cast<const uint4*>(src + j);  // may alias the output row: no __ldg
        const uint32_t w[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
        for (int e = 0; e < 8; ++e)
          v[j + e] += __uint_as_float((e & 1) ? (w[e >> 1] & 0xFFFF0000u) : (w[e >> 1] << 16));
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) v[j] += __bfloat162float(src[j]);
    }
  }
  if (ep.out_kind == kOutF32) {
    float* dst = reinterpret_cast<float*>(ep.out) + (long long)row * ep.ldo + col0;
    if (ep.vec_ok && col0 + 32 <= N) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) dst[j] = v[j];
    }
  } else {
    if (ep.row_amax) {
      float m = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) m = fmaxf(m, fabsf(bf16_round(v[j])));
      atomicMax(reinterpret_cast<int*>(ep.row_amax + row), __float_as_int(m));  // m >= 0: int order = float order
    }
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(ep.out) + (long long)row * ep.ldo + col0;
    if (ep.vec_ok && col0 + 32 <= N) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 p;
        p.x = pack_bf16(v[j], v[j + 1]);
        p.y = pack_bf16(v[j + 2], v[j + 3]);
        p.z = pack_bf16(v[j + 4], v[j + 5]);
        p.w = pack_bf16(v[j + 6], v[j + 7]);
        *reinterpret_cast<uint4*>(dst + j) = p;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) dst[j] = __float2bfloat16_rn(v[j]);
    }
  }
}

template <int KIND>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap ta2,
                const __grid_constant__ CUtensorMap tb, int M, int N, int K, int k_split, int kg,
                Epilogue ep, int* err) {
  using T = Traits<KIND>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* tfull = bars + 2 * kStages;
  uint64_t* tempty = bars + 2 * kStages + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = (N + BN - 1) / BN;
  const int total = num_m * num_n;
  const int nk = (K + T::BK - 1) / T::BK;  // the TMA zero-fills the K tail

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&tfull[a]), 1);
      mbar_init(smem_u32(&tempty[a]), kEpiWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch(&ta);
    tma_prefetch(&ta2);
    tma_prefetch(&tb);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    int stage = 0;
    uint32_t phase = 0;
    const int ks_blocks = (k_split + T::BK - 1) / T::BK;  // k-blocks read from the first A source
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      int m, n;
      tile_coords(t, num_m, num_n, m, n);
      bool ok = true;
      for (int kb = 0; kb < nk; ++kb) {
        if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1, abort_flag, err, kErrWaitProducer)) {
          ok = false;
          break;
        }
        const uint32_t sa = smem_u32(smem + stage * kStageBytes);
        const uint32_t sb = sa + kStageA;
        const uint32_t fb = smem_u32(&full[stage]);
        mbar_arrive_expect_tx(fb, kStageBytes);
        if (kg > 0)  // grouped K: A is [K / kg][M][kg], k-block kb lies inside one group
          tma_load_3d(sa, &ta, fb, (kb * T::BK) % kg, m * BM, (kb * T::BK) / kg);
        else if (kb < ks_blocks)
          tma_load_2d(sa, &ta, fb, kb * T::BK, m * BM);
        else
          tma_load_2d(sa, &ta2, fb, (kb - ks_blocks) * T::BK, m * BM);
        tma_load_2d(sb, &tb, fb, kb * T::BK, n * BN);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    int stage = 0;
    uint32_t phase = 0;
    int local = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1, abort_flag, err, kErrWaitMma)) break;
      tc_fence_after();
      const uint32_t d = tmem_base + acc * BN;
      bool ok = true;
      for (int kb = 0; kb < nk; ++kb) {
        if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, err, kErrWaitMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + stage * kStageBytes);
        const uint32_t sb = sa + kStageA;
#pragma unroll
        for (int k = 0; k < 128 / (T::UK * (KIND == 0 ? 2 : 1)); ++k) {
          const uint32_t koff = k * 32;  // 32 bytes of K per MMA
          T::mma(d, make_sdesc(sa + koff, 16, 1024), make_sdesc(sb + koff, 16, 1024),
                 (kb > 0 || k > 0) ? 1u : 0u);
        }
        tc_commit(smem_u32(&empty[stage]));
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      tc_commit(smem_u32(&tfull[acc]));
    }
  } else if (warp >= 2) {
    // ---------------- epilogue ----------------
    const int quad = warp & 3;  // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;  // which half of the tile's columns it drains
    const int row_in_tile = quad * 32 + lane;
    float alpha = ep.alpha;
    if (ep.dev_scale0) alpha *= *ep.dev_scale0;
    if (ep.dev_scale1) alpha *= *ep.dev_scale1;
    int local = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      int m, n;
      tile_coords(t, num_m, num_n, m, n);
      if (!mbar_wait(smem_u32(&tfull[acc]), acc_phase, abort_flag, err, kErrWaitEpilogue)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN;
      const int row = m * BM + row_in_tile;
      const int n0 = n * BN;
      const float ars = alpha * ((ep.row_scale && row < M) ? ep.row_scale[row] : 1.0f);
      uint32_t r[32];
      if (n0 < ep.norm_cols) {
        // q / k columns: raw bf16 + per-head RMSNorm into norm_out.
        const int hd = ep.head_dim;  // 64 or 128: each half of the tile holds whole heads
        for (int h0 = half * (BN / 2); h0 < (half + 1) * (BN / 2); h0 += hd) {
          const int c_head = n0 + h0;
          const float* w = ep.norm_w + (c_head < ep.norm_split ? 0 : hd);
          float ss = 0.f;
          for (int c = 0; c < hd; c += 32) {
            tmem_ld32(tbase + h0 + c, r);
            tmem_ld_wait();
            uint32_t pk[16];
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const float a = bf16_round(scaled<KIND>(ep, r[j], ars, c_head + c + j, N));
              const float b = bf16_round(scaled<KIND>(ep, r[j + 1], ars, c_head + c + j + 1, N));
              ss += a * a + b * b;
              pk[j / 2] = pack_bf16(a, b);
            }
            if (row < M) {
              __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(ep.out) + (long long)row * ep.ldo + c_head + c;
#pragma unroll
              for (int j = 0; j < 16; j += 4)
                *reinterpret_cast<uint4*>(dst + 2 * j) = make_uint4(pk[j], pk[j + 1], pk[j + 2], pk[j + 3]);
            }
          }
          const float inv = rsqrtf(ss / (float)hd + ep.eps);
          for (int c = 0; c < hd; c += 32) {
            tmem_ld32(tbase + h0 + c, r);
            tmem_ld_wait();
            uint32_t pk[16];
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const float a = bf16_round(scaled<KIND>(ep, r[j], ars, c_head + c + j, N)) * inv * w[c + j];
              const float b = bf16_round(scaled<KIND>(ep, r[j + 1], ars, c_head + c + j + 1, N)) * inv * w[c + j + 1];
              pk[j / 2] = pack_bf16(a, b);
            }
            if (row < M) {
              __nv_bfloat16* dst = ep.norm_out + (long long)row * ep.ld_norm + c_head + c;
#pragma unroll
              for (int j = 0; j < 16; j += 4)
                *reinterpret_cast<uint4*>(dst + 2 * j) = make_uint4(pk[j], pk[j + 1], pk[j + 2], pk[j + 3]);
            }
          }
          if (ep.act_out && c_head < ep.norm_split) {
            // branch q features of the video rows: silu(bf16 q) L2-normalised over the head,
            // stored frame-head-token-dim (kernels.py:47-51 with the FHSD permute)
            const int br = row - ep.act_row0;
            const bool mine = row < M && br >= 0 && br < ep.act_rows;
            float ss2 = 0.f;
            for (int c = 0; c < hd; c += 32) {
              tmem_ld32(tbase + h0 + c, r);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const float y = silu_fast(bf16_round(scaled<KIND>(ep, r[j], ars, c_head + c + j, N)));
                ss2 = fmaf(y, y, ss2);
              }
            }
            const float inv2 = 1.0f / fmaxf(sqrtf(ss2), 1e-6f);
            const int f = mine ? br / ep.act_tpf : 0, s = mine ? br - f * ep.act_tpf : 0;
            const int head = c_head / hd;
            __nv_bfloat16* dst = ep.act_out + (((long long)f * ep.act_heads + head) * ep.act_tpf + s) * hd;
            for (int c = 0; c < hd; c += 32) {
              tmem_ld32(tbase + h0 + c, r);
              tmem_ld_wait();
              uint32_t pk[16];
#pragma unroll
              for (int j = 0; j < 32; j += 2) {
                const float a = silu_fast(bf16_round(scaled<KIND>(ep, r[j], ars, c_head + c + j, N))) * inv2;
                const float b = silu_fast(bf16_round(scaled<KIND>(ep, r[j + 1], ars, c_head + c + j + 1, N))) * inv2;
                pk[j / 2] = pack_bf16(a, b);
              }
              if (mine) {
#pragma unroll
                for (int j = 0; j < 16; j += 4)
                  *reinterpret_cast<uint4*>(dst + c + 2 * j) = make_uint4(pk[j], pk[j + 1], pk[j + 2], pk[j + 3]);
              }
            }
          }
        }
      } else if (ep.act == kActSwiGLU) {
        // columns [n0, n0 + 128) hold the gate rows and [n0 + 128, n0 + 256) the matching up
        // rows of output columns [n0 / 2, n0 / 2 + 128) (the host interleaves W_fc1 that way):
        // out = silu(gate) * up with the reference's bf16 roundings (block_kernels.py:113-115)
        for (int c = half * (BN / 4); c < (half + 1) * (BN / 4); c += 32) {
          if (n0 + c >= N) break;
          uint32_t u[32];
          tmem_ld32(tbase + c, r);
          tmem_ld32(tbase + BN / 2 + c, u);
          tmem_ld_wait();
          if (row < M) {
            uint32_t pk[16];
            float m = 0.f;
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              float o[2];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int cg = n0 + c + j + e, cu = cg + BN / 2;
                float g = scaled<KIND>(ep, r[j + e], ars, cg, N), up = scaled<KIND>(ep, u[j + e], ars, cu, N);
                if (ep.col_bias) {
                  g += ep.col_bias[cg];
                  up += ep.col_bias[cu];
                }
                g = bf16_round(g);
                o[e] = bf16_round(g / (1.0f + __expf(-g))) * bf16_round(up);
                m = fmaxf(m, fabsf(bf16_round(o[e])));
              }
              pk[j / 2] = pack_bf16(o[0], o[1]);
            }
            if (ep.row_amax) atomicMax(reinterpret_cast<int*>(ep.row_amax + row), __float_as_int(m));
            __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(ep.out) + (long long)row * ep.ldo + n0 / 2 + c;
#pragma unroll
            for (int j = 0; j < 16; j += 4)
              *reinterpret_cast<uint4*>(dst + 2 * j) = make_uint4(pk[j], pk[j + 1], pk[j + 2], pk[j + 3]);
          }
        }
      } else {
        // 32-column chunks: a tile may straddle the v columns and the fp32 side columns
        for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += 32) {
          const int col = n0 + c;
          if (col >= N) break;
          tmem_ld32(tbase + c, r);
          tmem_ld_wait();
          if (ep.aux_out && col >= ep.aux_col0) {
            if (row < M) {
              float* dst = ep.aux_out + (long long)row * ep.ld_aux + (col - ep.aux_col0);
              const int lim = min(32, N - col);
              if (lim == 32) {
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                  *reinterpret_cast<float4*>(dst + j) =
                      make_float4(scaled<KIND>(ep, r[j], ars, col + j, N), scaled<KIND>(ep, r[j + 1], ars, col + j + 1, N),
                                  scaled<KIND>(ep, r[j + 2], ars, col + j + 2, N),
                                  scaled<KIND>(ep, r[j + 3], ars, col + j + 3, N));
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (j < lim) dst[j] = scaled<KIND>(ep, r[j], ars, col + j, N);
              }
            }
          } else {
            store_plain_chunk<KIND>(ep, r, row, col, M, N, alpha);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&tempty[acc]));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag) abort_drain();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256;

template <int KIND>
int launch(const void* A, long long lda, const void* A2, long long lda2, long long k_split,
           const void* B, long long ldb, int M, int N, int K, const Epilogue& ep, int* err,
           cudaStream_t stream, long long group_stride = 0, int kg = 0) {
  using T = Traits<KIND>;
  if (M <= 0 || N <= 0 || K <= 0 || (K % 16) != 0) return kUnsupported;
  if (kg > 0 && (A2 != nullptr || (kg % T::BK) != 0 || (K % kg) != 0)) return kUnsupported;
  if (A2 == nullptr) {
    A2 = A;
    lda2 = lda;
    k_split = K;
  }
  if (k_split <= 0 || k_split > K || (k_split != K && (k_split % T::BK) != 0)) return kUnsupported;
  const CUtensorMapDataType dt = KIND == 0 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const int eb = KIND == 0 ? 2 : 1;
  CUtensorMap ta, ta2, tb;
  int rc = kg > 0 ? make_tmap_3d(&ta, A, dt, eb, (uint64_t)kg, (uint64_t)M, (uint64_t)(K / kg), (uint64_t)lda,
                                 (uint64_t)group_stride, T::BK, BM)
                  : make_tmap_2d(&ta, A, dt, eb, (uint64_t)k_split, (uint64_t)M, (uint64_t)lda, T::BK, BM);
  if (rc) return rc;
  rc = make_tmap_2d(&ta2, A2, dt, eb, (uint64_t)(K - k_split > 0 ? K - k_split : T::BK), (uint64_t)M,
                    (uint64_t)lda2, T::BK, BM);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, B, dt, eb, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, T::BK, BN);
  if (rc) return rc;
  if (!smem_optin((const void*)gemm_kernel<KIND>, kSmemBytes)) return kLaunchFailed;
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int grid = tiles < sm_count() ? tiles : sm_count();
  gemm_kernel<KIND><<<grid, kThreads, kSmemBytes, stream>>>(ta, ta2, tb, M, N, K, (int)k_split, kg, ep, err);
  vdn::count_launch();
  return launch_status();
}

}  // namespace gemm
}  // namespace vdn

using vdn::gemm::Epilogue;

static Epilogue plain_epilogue(void* C, long long ldc, int out_kind, float alpha, const float* row_scale,
                               const float* col_scale, const float* col_bias, int act,
                               const void* addend, long long ld_add) {
  Epilogue ep{};
  ep.out = C;
  ep.ldo = ldc;
  ep.out_kind = out_kind;
  ep.act = act;
  ep.alpha = alpha;
  ep.row_scale = row_scale;
  ep.col_scale = col_scale;
  ep.col_bias = col_bias;
  ep.addend = reinterpret_cast<const __nv_bfloat16*>(addend);
  const long long ebytes = out_kind == vdn::gemm::kOutBF16 ? 2 : 4;
  ep.vec_ok = vdn::aligned16(C) && (ldc * ebytes) % 16 == 0;
  ep.ld_add = ld_add;
  ep.add_vec_ok = addend && vdn::aligned16(addend) && (ld_add * 2) % 16 == 0;
  ep.cs_vec_ok = col_scale && vdn::aligned16(col_scale);
  ep.cb_vec_ok = col_bias && vdn::aligned16(col_bias);
  ep.norm_cols = 0;
  ep.aux_col0 = 1 << 30;
  return ep;
}

extern "C" {

// C = epilogue(A * B^T) with kind 0 = bf16, 1 = fp8 e4m3, 2 = int8.  A may be split along K
// into two sources (A for k < k_split, A2 for the rest); pass A2 = NULL for one source.
int vdn_gemm(int kind, const void* A, long long lda, const void* A2, long long lda2, long long k_split,
             const void* B, long long ldb, void* C, long long ldc, int out_kind, int M, int N, int K,
             float alpha, const float* dev_scale0, const float* dev_scale1, const float* row_scale,
             const float* col_scale, const float* col_bias, int act, const void* addend, long long ld_add,
             int* dev_err, void* stream) {
  if (!A || !B || !C) return vdn::kBadArgument;
  if (out_kind == vdn::gemm::kOutS32 && kind != 2) return vdn::kBadArgument;
  if (act < vdn::gemm::kActNone || act > vdn::gemm::kActGelu) return vdn::kBadArgument;
  Epilogue ep = plain_epilogue(C, ldc, out_kind, alpha, row_scale, col_scale, col_bias, act, addend, ld_add);
  ep.dev_scale0 = dev_scale0;
  ep.dev_scale1 = dev_scale1;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (kind) {
    case 0: return vdn::gemm::launch<0>(A, lda, A2, lda2, k_split, B, ldb, M, N, K, ep, dev_err, s);
    case 1: return vdn::gemm::launch<1>(A, lda, A2, lda2, k_split, B, ldb, M, N, K, ep, dev_err, s);
    case 2: return vdn::gemm::launch<2>(A, lda, A2, lda2, k_split, B, ldb, M, N, K, ep, dev_err, s);
    default: return vdn::kBadArgument;
  }
}

// C = epilogue(A * B^T) with a grouped-K A operand: A holds `groups` slabs of [M, kg]
// (rows `lda` apart, slabs `group_stride` apart) and K = groups * kg runs through the
// slabs in order.  This reads an all-to-all receive buffer [ranks][rows][kg] directly
// as the K-concatenated operand of the row-split output projection.
int vdn_gemm_grouped_k(int kind, const void* A, long long lda, long long group_stride, int groups, int kg,
                       const void* B, long long ldb, void* C, long long ldc, int out_kind, int M, int N,
                       float alpha, const float* dev_scale0, const float* dev_scale1, const float* row_scale,
                       const float* col_scale, const float* col_bias, int act, const void* addend,
                       long long ld_add, int* dev_err, void* stream) {
  if (!A || !B || !C) return vdn::kBadArgument;
  if (groups <= 0 || kg <= 0) return vdn::kBadArgument;
  if (out_kind == vdn::gemm::kOutS32 && kind != 2) return vdn::kBadArgument;
  if (group_stride < (long long)M * lda) return vdn::kBadArgument;  // slabs must not overlap
  if (act < vdn::gemm::kActNone || act > vdn::gemm::kActGelu) return vdn::kBadArgument;
  Epilogue ep = plain_epilogue(C, ldc, out_kind, alpha, row_scale, col_scale, col_bias, act, addend, ld_add);
  ep.dev_scale0 = dev_scale0;
  ep.dev_scale1 = dev_scale1;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int K = groups * kg;
  switch (kind) {
    case 0: return vdn::gemm::launch<0>(A, lda, nullptr, 0, 0, B, ldb, M, N, K, ep, dev_err, s, group_stride, kg);
    case 1: return vdn::gemm::launch<1>(A, lda, nullptr, 0, 0, B, ldb, M, N, K, ep, dev_err, s, group_stride, kg);
    case 2: return vdn::gemm::launch<2>(A, lda, nullptr, 0, 0, B, ldb, M, N, K, ep, dev_err, s, group_stride, kg);
    default: return vdn::kBadArgument;
  }
}

// Fused QKV projection: one GEMM of x [S, hidden] against the concatenated weight
// [3*inner + n_aux, hidden] (q, k, v rows, then the fp32 side projections).
//   qkv_out  [S, 3*inner] bf16   raw q/k/v (hybrid.py:260-268)
//   qk_norm  [S, 2*inner] bf16   RMSNorm(q), RMSNorm(k) per head, weights norm_w[2, head_dim]
//   aux_out  [S, n_aux]   fp32   side projections (gate / beta / output-gate down / alpha down)
// kind: 0 bf16, 1 fp8 (per-tensor: alpha = s_x * s_w), 2 int8 (row_scale = per-token,
// col_scale = per-channel).
int vdn_qkv_gemm(int kind, const void* x, long long ldx, const void* w, long long ldw, int S, int hidden,
                 int inner, int n_aux, int head_dim, const float* norm_w, float eps, float alpha,
                 const float* dev_scale0, const float* dev_scale1, const float* row_scale,
                 const float* col_scale, void* qkv_out, long long ld_qkv, void* qk_norm, long long ld_norm,
                 float* aux_out, long long ld_aux, void* q_act, int act_row0, int act_rows, int act_tpf,
                 int* dev_err, void* stream) {
  if (!x || !w || !qkv_out || !qk_norm || !norm_w) return vdn::kBadArgument;
  // the QKV epilogue stores 16-byte vectors into all three outputs
  if (!vdn::aligned16(qkv_out) || !vdn::aligned16(qk_norm) || (ld_qkv * 2) % 16 || (ld_norm * 2) % 16 ||
      (aux_out && (!vdn::aligned16(aux_out) || (ld_aux * 4) % 16)))
    return vdn::kMisaligned;
  if (head_dim != 64 && head_dim != 128) return vdn::kUnsupported;
  // a 256-column tile never mixes normalised q/k columns with v or side columns
  if ((2 * inner) % vdn::gemm::BN != 0) return vdn::kUnsupported;
  if (n_aux > 0 && !aux_out) return vdn::kBadArgument;
  Epilogue ep = plain_epilogue(qkv_out, ld_qkv, vdn::gemm::kOutBF16, alpha, row_scale, col_scale, nullptr, 0,
                               nullptr, 0);
  ep.dev_scale0 = dev_scale0;
  ep.dev_scale1 = dev_scale1;
  ep.norm_cols = 2 * inner;
  ep.norm_split = inner;
  ep.head_dim = head_dim;
  ep.eps = eps;
  ep.norm_out = reinterpret_cast<__nv_bfloat16*>(qk_norm);
  ep.ld_norm = ld_norm;
  ep.norm_w = norm_w;
  ep.aux_col0 = 3 * inner;
  ep.aux_out = aux_out;
  ep.ld_aux = ld_aux;
  if (q_act) {
    // act_row0 is relative to this call's first row: a call over a block of rows (negative
    // act_row0 when the block starts inside the branch rows) writes the rows it holds
    if (!vdn::aligned16(q_act) || act_rows <= 0 || act_tpf <= 0 || act_rows % act_tpf) return vdn::kBadArgument;
    ep.act_out = reinterpret_cast<__nv_bfloat16*>(q_act);
    ep.act_row0 = act_row0;
    ep.act_rows = act_rows;
    ep.act_tpf = act_tpf;
    ep.act_heads = inner / head_dim;
  }
  const int N = 3 * inner + n_aux;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (kind) {
    case 0: return vdn::gemm::launch<0>(x, ldx, nullptr, 0, 0, w, ldw, S, N, hidden, ep, dev_err, s);
    case 1: return vdn::gemm::launch<1>(x, ldx, nullptr, 0, 0, w, ldw, S, N, hidden, ep, dev_err, s);
    case 2: return vdn::gemm::launch<2>(x, ldx, nullptr, 0, 0, w, ldw, S, N, hidden, ep, dev_err, s);
    default: return vdn::kBadArgument;
  }
}

// Block projections with the DiT pointwise work fused into the epilogue (block_kernels.py):
//   C[M, N'] bf16 = residual + gate[row_group[row]] * act(alpha * dev scales * row_scale * col_scale * (A B^T)
//                   + bias)
// act: 0 none, 2 GELU (erf), 3 SwiGLU over paired 128-row blocks of B (N' = N / 2, N % 256 == 0).
// A: one source (A2 = NULL, kg = 0), K-concatenated (A2 for k >= k_split) or grouped-K (kg > 0:
// `groups` = K / kg slabs `group_stride` apart).  residual [M, ld_res] bf16 and the gate table
// [groups of rows, ld_gate] bf16 with row_group [M] int32 are optional (both or neither gate).
// row_amax [M] fp32 (optional, zeroed by the caller) receives max |C[row, :]| of the stored values.
int vdn_gemm_block(int kind, const void* A, long long lda, const void* A2, long long lda2, long long k_split,
                   long long group_stride, int kg, const void* B, long long ldb, void* C, long long ldc, int M,
                   int N, int K, float alpha, const float* dev_scale0, const float* dev_scale1,
                   const float* row_scale, const float* col_scale, const float* col_bias, int act,
                   const void* residual, long long ld_res, const int* row_group, const void* group_gate,
                   long long ld_gate, float* row_amax, int* dev_err, void* stream) {
  if (!A || !B || !C) return vdn::kBadArgument;
  if (act != vdn::gemm::kActNone && act != vdn::gemm::kActGelu && act != vdn::gemm::kActSwiGLU)
    return vdn::kBadArgument;
  if ((row_group == nullptr) != (group_gate == nullptr)) return vdn::kBadArgument;
  if (act == vdn::gemm::kActSwiGLU) {
    // one tile = one gate block + its up block; the vector stores need 16-byte rows
    if (N % vdn::gemm::BN || group_gate || residual) return vdn::kUnsupported;
    if (!vdn::aligned16(C) || (ldc * 2) % 16) return vdn::kMisaligned;
  }
  if (kg > 0 && (A2 || group_stride < (long long)M * lda)) return vdn::kBadArgument;
  Epilogue ep = plain_epilogue(C, ldc, vdn::gemm::kOutBF16, alpha, row_scale, col_scale, col_bias, act, residual,
                               ld_res);
  ep.dev_scale0 = dev_scale0;
  ep.dev_scale1 = dev_scale1;
  ep.row_group = row_group;
  ep.group_gate = reinterpret_cast<const __nv_bfloat16*>(group_gate);
  ep.ld_group_gate = ld_gate;
  ep.row_amax = row_amax;
  ep.gate_vec_ok = group_gate && vdn::aligned16(group_gate) && (ld_gate * 2) % 16 == 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (kind) {
    case 0: return vdn::gemm::launch<0>(A, lda, A2, lda2, k_split, B, ldb, M, N, K, ep, dev_err, s, group_stride, kg);
    case 1: return vdn::gemm::launch<1>(A, lda, A2, lda2, k_split, B, ldb, M, N, K, ep, dev_err, s, group_stride, kg);
    case 2: return vdn::gemm::launch<2>(A, lda, A2, lda2, k_split, B, ldb, M, N, K, ep, dev_err, s, group_stride, kg);
    default: return vdn::kBadArgument;
  }
}

long long vdn_launch_count(void) { return vdn::launch_counter().load(std::memory_order_relaxed); }

}  // extern "C"
