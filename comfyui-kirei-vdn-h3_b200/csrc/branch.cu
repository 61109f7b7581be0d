// Video Delta Attention (VDA) linear branch of VDN-H3 on sm_100a.
//
// Pipeline for the F' = F-2 inner frames of one block (branch.py:672-816, runtime.py:545-607):
//   1. vdn_spatial_conv   depthwise kxk conv per frame on the (gh, gw) grid      (branch.py:469-471)
//   2. vdn_temporal_act   5-tap temporal conv (zero pad), SiLU, L2 over D, FHSD  (kernels.py:99-129)
//                         (taps = 0: plain activation for q and text rows, kernels.py:47-51)
//   3. vdn_alpha_gate     alpha = exp(-exp(A_log) softplus(up(mean_t down x) + dt_bias)) (branch.py:483-491)
//   4. vdn_frame_stats    A = sym((beta K)^T K), B = (beta V)^T K per frame/head  (branch.py:197-243)
//   5. vdn_delta_factor   (I+A)^-1 of every SPD frame matrix, leading-minor info (branch.py:148-160, :62-71)
//   6. vdn_bidir_scan     s_t = (B_t + s_{t-1} diag(alpha_t)) (I+A_t)^-1, both directions
//                         (= Inj_t + s_{t-1} T_t of branch.py:297-312, fused so neither T nor
//                          Inj is ever materialised)
//   7. vdn_readout        gather + alpha bridge (branch.py:372-396), Q S^T, RMSNorm(D),
//                         x output gate (branch.py:494-530, :754-758)
// Every kernel reads and writes device buffers through plain pointers and strides.
#include "host_common.h"
#include "sm100.cuh"

namespace vdn {
namespace branch {

// x * sigmoid(x) = x / (1 + 2^(-x log2 e)) with the hardware's approximate exp2 and
// reciprocal (2 ulp; the result is rounded to bf16), in their flush-to-zero forms, which
// skip the subnormal handling (a subnormal intermediate becomes 0); for x -> -inf the
// denominator overflows to inf, its reciprocal is 0 and the product -0
__device__ __forceinline__ float silu(float x) { return x * rcp_ftz(1.0f + ex2_ftz(-x * 1.4426950408889634f)); }
__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + __expf(-x)); }
__device__ __forceinline__ float softplusf_(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

// ---------------------------------------------------------------------------------
// 1. Spatial depthwise 5x5 conv.  in: rows (f*gh + y)*gw + x at row pitch ld_in; out
// [rows, C] bf16 (rounded like the reference's bf16 conv2d output).
// One thread per (channel pair, grid row); it slides along x keeping the 5x5 window of
// both channels in registers, so each output costs 5 paired loads and 50 FMAs.
// grid (ceil(C/256), gh, F), block 128.
// ---------------------------------------------------------------------------------
__global__ void __launch_bounds__(128) spatial_conv5_kernel(const __nv_bfloat16* __restrict__ in, long long ld_in,
                                                            const float* __restrict__ w, int gh, int gw, int C,
                                                            __nv_bfloat16* __restrict__ out, long long ld_out) {
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 2;
  const int y = blockIdx.y, f = blockIdx.z;
  if (c >= C) return;
  float2 wr[5][5];
#pragma unroll
  for (int dy = 0; dy < 5; ++dy)
#pragma unroll
    for (int dx = 0; dx < 5; ++dx)
      wr[dy][dx] = make_float2(w[(long long)c * 25 + dy * 5 + dx], w[(long long)(c + 1) * 25 + dy * 5 + dx]);
  const long long frame0 = (long long)f * gh * gw;
  auto load_col = [&](int x, float2 (&col)[5]) {
#pragma unroll
    for (int dy = 0; dy < 5; ++dy) {
      const int yy = y + dy - 2;
      if (x >= 0 && x < gw && yy >= 0 && yy < gh) {
        const __nv_bfloat162 v =
            *reinterpret_cast<const __nv_bfloat162*>(in + (frame0 + (long long)yy * gw + x) * ld_in + c);
        col[dy] = __bfloat1622float2(v);
      } else {
        col[dy] = make_float2(0.f, 0.f);
      }
    }
  };
  float2 win[5][5];  // win[slot][dy]; slot (u + k) % 5 holds column x - 2 + k
#pragma unroll
  for (int s = 0; s < 5; ++s) load_col(s - 2, win[s]);
  for (int x0 = 0; x0 < gw; x0 += 5) {
#pragma unroll
    for (int u = 0; u < 5; ++u) {
      const int x = x0 + u;
      if (x < gw) {
        float2 acc = make_float2(0.f, 0.f);
#pragma unroll
        for (int k = 0; k < 5; ++k)
#pragma unroll
          for (int dy = 0; dy < 5; ++dy) {
            acc.x += wr[dy][k].x * win[(u + k) % 5][dy].x;
            acc.y += wr[dy][k].y * win[(u + k) % 5][dy].y;
          }
        *reinterpret_cast<__nv_bfloat162*>(out + (frame0 + (long long)y * gw + x) * ld_out + c) =
            __floats2bfloat162_rn(acc.x, acc.y);
        load_col(x + 3, win[u]);  // replaces column x - 2
      }
    }
  }
}

// Tiled 5x5 depthwise conv.  A persistent CTA of four warps walks a contiguous range of
// tiles (64 channels x 8 output rows of one frame, channel-slab-major so the weights
// change rarely).  Each tile's input rows y0-2 .. y0+9 are staged in shared memory by
// 16-byte cp.async copies, the zero padding (two columns left and right, rows outside the
// frame) by the zero-filling form of the same copy, so the inner loop has no bounds
// checks.  Several CTAs share an SM (four at config 1, where registers rather than the
// 40 KB buffers set the count), so the copies of some are in flight while the others
// compute.
// Warp w computes output rows y0 + 2w, y0 + 2w + 1, lane l channels c0 + 2l, 2l + 1.  It
// walks the staged columns left to right: the 6 rows of a column are read once and added
// into every output they feed (2 rows x 5 columns of running paired-fp32 sums in
// registers), and the output column that the column completes is stored.  Per output
// that is 25 paired FMAs, 3 paired shared loads and one 4-byte store, against 5 loads and
// 4 extra adds when each output gathers its own 5x5 window.  At config 1 (29 frames of
// 38 x 22, 5120 channels) this runs in 253 us against 329 us for one warp per output row
// gathering its window (281 us with a staging loop that recomputed each copy's row and
// column); on the transposed 22 x 38 grid 4 rows per warp (two-warp CTAs, fewer warps per
// SM) took 402 us against 279 us for 2.
constexpr int kConvRows = 8;         // output rows per tile
constexpr int kConvWarpRows = 2;     // output rows per warp
constexpr int kConvCh = 64;          // channels per tile: two per lane
constexpr int kConvThreads = kConvRows / kConvWarpRows * 32;
constexpr int kConvMaxCtas = 3;      // CTAs per SM the register budget is sized for

__device__ __forceinline__ float2 lds_bf162(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}

__global__ void __launch_bounds__(kConvThreads, kConvMaxCtas)
    spatial_conv5_tiled_kernel(const __nv_bfloat16* __restrict__ in, long long ld_in, const float* __restrict__ w,
                               int F, int gh, int gw, int C, __nv_bfloat16* __restrict__ out, long long ld_out) {
  extern __shared__ __align__(16) __nv_bfloat16 conv_smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bands = (gh + kConvRows - 1) / kConvRows;
  const int per_slab = F * bands;
  const int n_tiles = (C / kConvCh) * per_slab;
  const int pitch = gw + 4;  // shared-memory columns per row: image column x sits at x + 2
  const int t0 = (int)((long long)blockIdx.x * n_tiles / gridDim.x);
  const int t1 = (int)((long long)(blockIdx.x + 1) * n_tiles / gridDim.x);
  if (t0 >= t1) return;

  // Thread tid copies the (staged column, 16-byte chunk of 8 channels) pairs p = tid,
  // tid + kConvThreads, ... < pitch * 8, each down all kConvRows + 4 staged rows: per copy
  // only the row's bounds bit and one address step change.
  const long long row_pitch = (long long)gw * ld_in;  // one image row down
  auto issue = [&](int t) {
    const int slab = t / per_slab, r = t - slab * per_slab;
    const int f = r / bands, y0 = (r - f * bands) * kConvRows;
    const __nv_bfloat16* frame = in + (long long)f * gh * gw * ld_in + slab * kConvCh;
    uint32_t rows_in = 0;  // bit i: staged row i lies inside the frame (the same for every thread)
#pragma unroll
    for (int i = 0; i < kConvRows + 4; ++i) rows_in |= (y0 - 2 + i >= 0 && y0 - 2 + i < gh) ? 1u << i : 0u;
    for (int p = tid; p < pitch * 8; p += kConvThreads) {
      const int col = p >> 3, q = p & 7, xx = col - 2;
      const bool col_in = xx >= 0 && xx < gw;
      const __nv_bfloat16* src = frame + ((long long)(y0 - 2) * gw + xx) * ld_in + q * 8;
      uint32_t dst = smem_u32(conv_smem + col * kConvCh + q * 8);
#pragma unroll 4
      for (int i = 0; i < kConvRows + 4; ++i, src += row_pitch, dst += pitch * kConvCh * 2) {
        const bool inside = col_in && ((rows_in >> i) & 1u);
        // padding positions read nothing (zero fill) from the frame's first pixel
        cp_async16_zfill(dst, inside ? src : frame, inside ? 16u : 0u);
      }
    }
    cp_async_commit();
  };

  float2 wr[5][5];
  int cur_slab = -1;
  for (int t = t0; t < t1; ++t) {
    issue(t);
    cp_async_wait<0>();
    __syncthreads();
    const int slab = t / per_slab, r = t - slab * per_slab;
    const int f = r / bands, y0 = (r - f * bands) * kConvRows;
    const int c = slab * kConvCh + 2 * lane;
    if (slab != cur_slab) {
#pragma unroll
      for (int dy = 0; dy < 5; ++dy)
#pragma unroll
        for (int dx = 0; dx < 5; ++dx)
          wr[dy][dx] = make_float2(w[(long long)c * 25 + dy * 5 + dx], w[(long long)(c + 1) * 25 + dy * 5 + dx]);
      cur_slab = slab;
    }
    const int y = y0 + warp * kConvWarpRows;
    if (y < gh) {
      const int rows = min(kConvWarpRows, gh - y);
      // shared row warp * kConvWarpRows + i holds image row y - 2 + i (zeros outside the frame)
      const __nv_bfloat16* base = conv_smem + warp * kConvWarpRows * pitch * kConvCh + 2 * lane;
      __nv_bfloat16* orow = out + (long long)(f * gh + y) * gw * ld_out + c;
      float2 acc[5][kConvWarpRows];  // acc[x % 5][o]: the running sum of output (y + o, x)
#pragma unroll
      for (int k = 0; k < 5; ++k)
#pragma unroll
        for (int o = 0; o < kConvWarpRows; ++o) acc[k][o] = make_float2(0.f, 0.f);
      // staged column s (image column s - 2, s % 5 == u) feeds output x = s - dx through
      // kernel column dx; the sum of x starts at dx = 0 and is complete after dx = 4
      auto column = [&](int s, int u) {
        float2 v[kConvWarpRows + 4];
#pragma unroll
        for (int i = 0; i < kConvWarpRows + 4; ++i) v[i] = lds_bf162(base + (i * pitch + s) * kConvCh);
#pragma unroll
        for (int dx = 0; dx < 5; ++dx) {
          const int k = (u - dx + 5) % 5;
#pragma unroll
          for (int o = 0; o < kConvWarpRows; ++o)
#pragma unroll
            for (int dy = 0; dy < 5; ++dy)
              acc[k][o] = (dx == 0 && dy == 0) ? mul2(wr[0][0], v[o]) : fma2(wr[dy][dx], v[o + dy], acc[k][o]);
        }
        const int x = s - 4;
        if (x >= 0) {
          const int k = (u + 1) % 5;
#pragma unroll
          for (int o = 0; o < kConvWarpRows; ++o)
            if (o < rows)
              *reinterpret_cast<__nv_bfloat162*>(orow + ((long long)o * gw + x) * ld_out) =
                  __floats2bfloat162_rn(acc[k][o].x, acc[k][o].y);
        }
      };
      int s0 = 0;
      for (; s0 + 5 <= pitch; s0 += 5) {
#pragma unroll
        for (int u = 0; u < 5; ++u) column(s0 + u, u);
      }
#pragma unroll
      for (int u = 0; u < 5; ++u)
        if (s0 + u < pitch) column(s0 + u, u);
    }
    __syncthreads();  // every warp is done with the buffer before it is refilled
  }
}

// Generic odd kernel sizes (kh*kw <= 49): one thread per channel, direct sum.
__global__ void spatial_conv_kernel(const __nv_bfloat16* __restrict__ in, long long ld_in,
                                    const float* __restrict__ w, int kh, int kw, int gh, int gw, int C,
                                    __nv_bfloat16* __restrict__ out, long long ld_out) {
  const int y = blockIdx.x, f = blockIdx.y;
  const int c = blockIdx.z * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int taps = kh * kw;
  const int ph = kh / 2, pw = kw / 2;
  const long long frame0 = (long long)f * gh * gw;
  for (int x = 0; x < gw; ++x) {
    float acc = 0.f;
    for (int dy = 0; dy < kh; ++dy) {
      const int yy = y + dy - ph;
      if (yy < 0 || yy >= gh) continue;
      for (int dx = 0; dx < kw; ++dx) {
        const int xx = x + dx - pw;
        if (xx < 0 || xx >= gw) continue;
        acc += w[(long long)c * taps + dy * kw + dx] * __bfloat162float(in[(frame0 + (long long)yy * gw + xx) * ld_in + c]);
      }
    }
    out[(frame0 + (long long)y * gw + x) * ld_out + c] = __float2bfloat16_rn(acc);
  }
}

// ---------------------------------------------------------------------------------
// 2. Temporal conv + SiLU + optional L2, output FHSD [F, H, T, D] bf16.
// One warp per (token s, head h); lane l holds channels h*D + l*D/32 .. +D/32 as fp32
// pairs.  The warp walks the frames keeping the next 4 input frames in flight (one 8-byte
// load per lane and frame for D = 128): each output unpacks one of them into a sliding
// window of 5, reloads its slot with the frame 4 outputs ahead, and runs the 5-tap conv
// (paired FMAs), SiLU and the L2 norm (a warp reduction) from registers, so every input
// frame is unpacked once.  taps 0 (no temporal conv), 1 and 3 run with a window of 1 or 3.
// Config 1 (k, 5 taps + L2): 136 us with 4 frames in flight, 142 / 152 us with 3 / 2, 177 us
// with 8 (which spills at this register budget); loading 8 frames per 8-output chunk only
// after the previous chunk took 152 us.
// ---------------------------------------------------------------------------------
template <int V>
struct PackedBf16;
template <>
struct PackedBf16<4> {
  using T = uint2;
  __device__ static void unpack2(T p, float2 (&v)[2]) {
    v[0] = make_float2(__uint_as_float(p.x << 16), __uint_as_float(p.x & 0xffff0000u));
    v[1] = make_float2(__uint_as_float(p.y << 16), __uint_as_float(p.y & 0xffff0000u));
  }
  __device__ static T pack2(const float2 (&v)[2]) {
    return make_uint2(pack_bf16(v[0].x, v[0].y), pack_bf16(v[1].x, v[1].y));
  }
};
template <>
struct PackedBf16<2> {
  using T = uint32_t;
  __device__ static void unpack2(T p, float2 (&v)[1]) {
    v[0] = make_float2(__uint_as_float(p << 16), __uint_as_float(p & 0xffff0000u));
  }
  __device__ static T pack2(const float2 (&v)[1]) { return pack_bf16(v[0].x, v[0].y); }
};

template <int D, int TAPS>
__global__ void __launch_bounds__(256, 3) temporal_act_kernel(const __nv_bfloat16* __restrict__ in, long long ld_in,
                                                           const float* __restrict__ w, int taps, int F, int T,
                                                           int H, int l2, __nv_bfloat16* __restrict__ out) {
  constexpr int V = D / 32;    // channels per lane
  constexpr int NP = V / 2;    // fp32 pairs per lane
  constexpr int kChunk = 4;    // input frames in flight (the unroll of the output loop)
  constexpr int kPad = TAPS / 2;
  using P = PackedBf16<V>;
  const int gwarp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gwarp >= T * H) return;
  const int s = gwarp / H, h = gwarp % H;
  const int c0 = h * D + lane * V;
  // y_t = sum_dt wt[dt] x_{t - pad + dt}, frames outside [0, F) are zero; no conv
  // (taps == 0) = one tap of weight 1
  float2 wt[TAPS][NP];
#pragma unroll
  for (int dt = 0; dt < TAPS; ++dt)
#pragma unroll
    for (int p = 0; p < NP; ++p)
      wt[dt][p] = taps == 0 ? make_float2(1.f, 1.f)
                            : make_float2(w[(long long)(c0 + 2 * p) * taps + dt], w[(long long)(c0 + 2 * p + 1) * taps + dt]);
  const __nv_bfloat16* src = in + (long long)s * ld_in + c0;
  const long long frame_pitch = (long long)T * ld_in;
  auto load = [&](int tt) {
    typename P::T r{};
    if (tt >= 0 && tt < F) r = *reinterpret_cast<const typename P::T*>(src + tt * frame_pitch);
    return r;
  };
  __nv_bfloat16* dst = out + ((long long)h * T + s) * D + lane * V;
  const long long out_pitch = (long long)H * T * D;
  // win[j] = frame t - pad + j while output t is computed; before output 0 the frames
  // -pad .. pad - 1 sit in win[1 ..], and each output shifts the window by one frame
  float2 win[TAPS][NP];
#pragma unroll
  for (int j = 1; j < TAPS; ++j) P::unpack2(load(j - kPad - 1), win[j]);
  // raw[i]: the frame entering the window at output t0 + i; once unpacked, its slot is
  // refilled with the frame output t0 + i + kChunk needs, so loads stay in flight throughout
  typename P::T raw[kChunk];
#pragma unroll
  for (int i = 0; i < kChunk; ++i) raw[i] = load(i + kPad);
  for (int t0 = 0; t0 < F; t0 += kChunk) {
#pragma unroll
    for (int i = 0; i < kChunk; ++i) {
      const int t = t0 + i;
      if (t >= F) break;
#pragma unroll
      for (int j = 0; j + 1 < TAPS; ++j)
#pragma unroll
        for (int p = 0; p < NP; ++p) win[j][p] = win[j + 1][p];
      P::unpack2(raw[i], win[TAPS - 1]);
      raw[i] = load(t + kChunk + kPad);
      float2 y[NP];
#pragma unroll
      for (int p = 0; p < NP; ++p) y[p] = fma2(wt[0][p], win[0][p], make_float2(0.f, 0.f));
#pragma unroll
      for (int dt = 1; dt < TAPS; ++dt)
#pragma unroll
        for (int p = 0; p < NP; ++p) y[p] = fma2(wt[dt][p], win[dt][p], y[p]);
      float ss = 0.f;
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        y[p].x = silu(y[p].x);
        ss += y[p].x * y[p].x;
        y[p].y = silu(y[p].y);
        ss += y[p].y * y[p].y;
      }
      if (l2) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        // 1 / max(|y|, 1e-6) = rsqrt(max(|y|^2, 1e-12)), by the hardware's approximate
        // reciprocal square root (2 ulp, far below the bf16 rounding of the output)
        const float inv = rsqrt_ftz(fmaxf(ss, 1e-12f));
#pragma unroll
        for (int p = 0; p < NP; ++p) y[p] = make_float2(y[p].x * inv, y[p].y * inv);
      }
      *reinterpret_cast<typename P::T*>(dst + t * out_pitch) = P::pack2(y);
    }
  }
}

// ---------------------------------------------------------------------------------
// 1+2 fused: the short conv features in one pass over the raw projection (branch.py:443-480
// with kernels.py:99-129): depthwise 5x5 spatial conv per frame (bf16-rounded, as the
// reference's bf16 conv2d output), 5-tap temporal conv (zero padded at the clip ends),
// SiLU, optional L2 over the head, FHSD output.  The same arithmetic, in the same order, as
// vdn_spatial_conv followed by vdn_temporal_act, without the intermediate round trip
// through HBM.
//
// A unit is one head (D channels) x 4 output rows x up to kFeatMaxCols output columns of
// the frame grid, walked through every frame in order: frame t's input rows (with a 2-pixel
// zero-padded halo) are staged in shared memory by cp.async while frame t-1 is computed;
// each thread computes its row's spatial outputs for two channels (the sliding 5x5 window of
// spatial_conv5_tiled_kernel) into a 5-frame ring in shared memory, which only that thread
// reads back: the temporal output of frame t-2 combines ring slots t-4 .. t.  Warp w owns
// row w % 4 and channels 64 (w / 4) + 2 lane, +1; the L2 sum of a position spans the
// D / 64 warps of its row (exchanged through shared memory) and is reduced in the tree of
// vdn_temporal_act's 32 lanes of D / 32 channels.  Units are ordered head by head, band by
// band, so neighbouring bands run at the same time and their shared halo rows come from L2.
// ---------------------------------------------------------------------------------
constexpr int kFeatRows = 4;
constexpr int kFeatMaxCols = 22;  // two staging buffers, the ring and the L2 exchange fit 227 KB at D = 128

template <int D>
struct FeatLayout {
  static constexpr int kHalves = D / 64;
  static constexpr int kThreads = 128 * kHalves;
  __host__ __device__ static int stage_elems(int wc) { return (kFeatRows + 4) * (wc + 4) * D; }
  __host__ __device__ static int ring_elems(int wc) { return 5 * kFeatRows * wc * D; }
  __host__ __device__ static size_t bytes(int wc) {
    return (size_t)(2 * stage_elems(wc) + ring_elems(wc)) * 2 + (size_t)kFeatRows * kHalves * kFeatMaxCols * 16 * 4;
  }
};

template <int D>
__global__ void __launch_bounds__(FeatLayout<D>::kThreads, 1)
    conv_features_kernel(const __nv_bfloat16* __restrict__ in, long long ld_in, const float* __restrict__ w_sp,
                         const float* __restrict__ w_tm, int F, int gh, int gw, int H, int wc, int l2,
                         __nv_bfloat16* __restrict__ out) {
  using L = FeatLayout<D>;
  extern __shared__ __align__(16) __nv_bfloat16 feat_smem[];
  __nv_bfloat16* stage = feat_smem;                     // [2][rows + 4][wc + 4][D]
  __nv_bfloat16* ring = feat_smem + 2 * L::stage_elems(wc);  // [5][rows][wc][D]
  float* part = reinterpret_cast<float*>(ring + L::ring_elems(wc));  // [rows][halves][kFeatMaxCols][16]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = warp & (kFeatRows - 1), hh = warp / kFeatRows;
  const int T = gh * gw;
  const int pitch = wc + 4;
  const int bands = (gh + kFeatRows - 1) / kFeatRows;
  const int cblocks = (gw + wc - 1) / wc;
  const int n_units = H * bands * cblocks;
  const int cl = hh * 64 + 2 * lane;  // this thread's first channel inside the head

  for (int unit = blockIdx.x; unit < n_units; unit += gridDim.x) {
    const int h = unit / (bands * cblocks);
    const int rem = unit - h * bands * cblocks;
    const int band = rem / cblocks, cb = rem - band * cblocks;
    const int y0 = band * kFeatRows, x0 = cb * wc;
    const int ncols = min(wc, gw - x0);
    const bool row_on = y0 + r < gh;
    const int c = h * D + cl;  // global channel
    float2 wr[5][5];
#pragma unroll
    for (int dy = 0; dy < 5; ++dy)
#pragma unroll
      for (int dx = 0; dx < 5; ++dx)
        wr[dy][dx] = make_float2(w_sp[(long long)c * 25 + dy * 5 + dx], w_sp[(long long)(c + 1) * 25 + dy * 5 + dx]);
    float2 wt[5];
#pragma unroll
    for (int dt = 0; dt < 5; ++dt) wt[dt] = make_float2(w_tm[(long long)c * 5 + dt], w_tm[(long long)(c + 1) * 5 + dt]);

    auto issue = [&](int f, int buf) {
      __nv_bfloat16* dst0 = stage + buf * L::stage_elems(wc);
      constexpr int kChunks = D / 8;  // 16-byte pieces of one pixel's D channels
      const int total = (kFeatRows + 4) * pitch * kChunks;
      for (int i = tid; i < total; i += L::kThreads) {
        const int q = i % kChunks, px = i / kChunks;
        const int row = px / pitch, col = px - row * pitch;
        const int yy = y0 - 2 + row, xx = x0 + col - 2;
        __nv_bfloat16* dst = dst0 + px * D + q * 8;
        if (yy >= 0 && yy < gh && xx >= 0 && xx < gw && col < ncols + 4)
          cp_async16(smem_u32(dst), in + ((long long)(f * gh + yy) * gw + xx) * ld_in + h * D + q * 8);
        else
          *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
      }
      cp_async_commit();
    };
    // this thread's ring entries: frames before the clip read as zeros
    __nv_bfloat16* my_ring = ring + (r * wc) * D + cl;  // + slot * rows * wc * D + x * D
    const int slot_stride = kFeatRows * wc * D;
    for (int s = 0; s < 5; ++s)
      for (int x = 0; x < ncols; ++x)
        *reinterpret_cast<uint32_t*>(my_ring + s * slot_stride + x * D) = 0u;

    issue(0, 0);
    for (int t = 0; t < F + 2; ++t) {
      const int slot = t % 5;
      if (t < F) {
        if (t + 1 < F) {
          issue(t + 1, (t + 1) & 1);
          cp_async_wait<1>();
        } else {
          cp_async_wait<0>();
        }
        __syncthreads();
        if (row_on) {
          // shared row r + dy holds image row y0 + r - 2 + dy; shared column x + k image column x0 + x - 2 + k
          const __nv_bfloat16* base = stage + (t & 1) * L::stage_elems(wc) + r * pitch * D + cl;
          __nv_bfloat16* wring = my_ring + slot * slot_stride;
          float2 win[5][5];  // win[slot][dy]; slot (x + k) % 5 holds shared column x + k
#pragma unroll
          for (int s = 0; s < 5; ++s)
#pragma unroll
            for (int dy = 0; dy < 5; ++dy) win[s][dy] = lds_bf162(base + (dy * pitch + s) * D);
          auto step = [&](int u, int x) {
            float2 a[5];
#pragma unroll
            for (int dy = 0; dy < 5; ++dy) a[dy] = make_float2(0.f, 0.f);
#pragma unroll
            for (int k = 0; k < 5; ++k)
#pragma unroll
              for (int dy = 0; dy < 5; ++dy) a[dy] = fma2(wr[dy][k], win[(u + k) % 5][dy], a[dy]);
            const float2 sum = add2(add2(add2(a[0], a[1]), add2(a[2], a[3])), a[4]);
            *reinterpret_cast<__nv_bfloat162*>(wring + x * D) = __floats2bfloat162_rn(sum.x, sum.y);
            if (x + 5 < pitch) {
#pragma unroll
              for (int dy = 0; dy < 5; ++dy) win[u][dy] = lds_bf162(base + (dy * pitch + x + 5) * D);
            }
          };
          int x = 0;
          for (; x + 5 <= ncols; x += 5) {
#pragma unroll
            for (int u = 0; u < 5; ++u) step(u, x + u);
          }
#pragma unroll
          for (int u = 0; u < 5; ++u)
            if (x + u < ncols) step(u, x + u);
        }
      } else {
        // frames past the clip read as zeros
        for (int x = 0; x < ncols; ++x) *reinterpret_cast<uint32_t*>(my_ring + slot * slot_stride + x * D) = 0u;
      }
      if (t >= 2) {
        // temporal conv of frame fo = t - 2 over slots fo - 2 .. fo + 2, then SiLU and the L2 sum
        const int fo = t - 2;
        float2 y[kFeatMaxCols];
        float ssq[kFeatMaxCols];
#pragma unroll
        for (int x = 0; x < kFeatMaxCols; ++x) {
          if (x < ncols) {
            float2 acc = make_float2(0.f, 0.f);
#pragma unroll
            for (int dt = 0; dt < 5; ++dt) {
              const float2 v = lds_bf162(my_ring + ((fo + 3 + dt) % 5) * slot_stride + x * D);  // frame fo - 2 + dt
              acc.x = fmaf(wt[dt].x, v.x, acc.x);
              acc.y = fmaf(wt[dt].y, v.y, acc.y);
            }
            y[x] = make_float2(silu(acc.x), silu(acc.y));
            // vdn_temporal_act's lane sum over D / 32 consecutive channels, in order
            float s = fmaf(y[x].y, y[x].y, y[x].x * y[x].x);
            if (D == 128) {  // lanes 2m, 2m + 1 hold the four channels of one such sum
              const float lo = __shfl_xor_sync(0xffffffffu, s, 1);
              const float2 yo = make_float2(__shfl_xor_sync(0xffffffffu, y[x].x, 1),
                                            __shfl_xor_sync(0xffffffffu, y[x].y, 1));
              s = (lane & 1) ? fmaf(y[x].y, y[x].y, fmaf(y[x].x, y[x].x, lo))
                             : fmaf(yo.y, yo.y, fmaf(yo.x, yo.x, s));
            }
            ssq[x] = s;
          }
        }
        if (l2) {
          if (D == 128) {
            // the tree's first step pairs sums of the row's two warps (channels c and c + 64):
            // one value per lane pair and position goes through shared memory
            float* mine = part + ((r * L::kHalves + hh) * kFeatMaxCols) * 16 + (lane >> 1);
            const float* theirs = part + ((r * L::kHalves + (hh ^ 1)) * kFeatMaxCols) * 16 + (lane >> 1);
            if ((lane & 1) == 0) {
#pragma unroll
              for (int x = 0; x < kFeatMaxCols; ++x)
                if (x < ncols) mine[x * 16] = ssq[x];
            }
            asm volatile("bar.sync %0, %1;" ::"r"(1 + r), "n"(64) : "memory");  // the row's two warps
#pragma unroll
            for (int x = 0; x < kFeatMaxCols; ++x)
              if (x < ncols) ssq[x] += theirs[x * 16];
          }
#pragma unroll
          for (int x = 0; x < kFeatMaxCols; ++x) {
            if (x < ncols) {
              float s = ssq[x];
#pragma unroll
              // the remaining steps inside the warp (lane pairs share a value at D = 128)
              for (int o = 16; o >= (D == 128 ? 2 : 1); o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
              const float inv = rsqrt_ftz(fmaxf(s, 1e-12f));  // as temporal_act_kernel
              y[x].x *= inv;
              y[x].y *= inv;
            }
          }
        }
        if (row_on) {
          const int s0 = (y0 + r) * gw + x0;
          __nv_bfloat16* orow = out + (((long long)fo * H + h) * T + s0) * D + cl;
#pragma unroll
          for (int x = 0; x < kFeatMaxCols; ++x)
            if (x < ncols) *reinterpret_cast<__nv_bfloat162*>(orow + (long long)x * D) = __floats2bfloat162_rn(y[x].x, y[x].y);
        }
      }
      __syncthreads();  // the stage buffer refilled next is free
    }
  }
}

// ---------------------------------------------------------------------------------
// 3. alpha gate.  down[rows, ld_down] fp32 (the x W_down^T columns, computed by the
// projection GEMM), mean over the T rows of each frame, then up + dt_bias, softplus.
// grid F, block 256.  alpha out [F, H, D] fp32.
// ---------------------------------------------------------------------------------
constexpr int kAlphaThreads = 512;

__global__ void __launch_bounds__(kAlphaThreads) alpha_gate_kernel(const float* __restrict__ down, long long ld_down,
                                                                   int T, int R, const float* __restrict__ w_up,
                                                                   const float* __restrict__ dt_bias,
                                                                   const float* __restrict__ a_log, int H, int D,
                                                                   float* __restrict__ alpha) {
  extern __shared__ float mean[];  // [R] then [kAlphaThreads] partials
  float* part = mean + R;
  const int f = blockIdx.x;
  // frame mean: G = kAlphaThreads / Rc row phases per column chunk of Rc columns; each
  // thread keeps 8 independent partial sums so 8 loads are in flight
  const int Rc = R < kAlphaThreads ? R : kAlphaThreads;
  const int G = kAlphaThreads / Rc;
  for (int j0 = 0; j0 < R; j0 += Rc) {
    const int j = j0 + (int)threadIdx.x % Rc, r0 = (int)threadIdx.x / Rc;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (j < R && r0 < G) {
      const float* col = down + (long long)f * T * ld_down + j;
      int s = r0;
      for (; s + 7 * G < T; s += 8 * G) {
#pragma unroll
        for (int u = 0; u < 8; ++u) acc[u] += col[(long long)(s + u * G) * ld_down];
      }
      for (; s < T; s += G) acc[0] += col[(long long)s * ld_down];
    }
    part[threadIdx.x] = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
    __syncthreads();
    if ((int)threadIdx.x < Rc && j0 + (int)threadIdx.x < R) {
      float tot = 0.f;
      for (int r = 0; r < G; ++r) tot += part[r * Rc + threadIdx.x];
      mean[j0 + threadIdx.x] = tot / (float)T;
    }
    __syncthreads();
  }
  const int inner = H * D;
  for (int c = blockIdx.y * blockDim.x + threadIdx.x; c < inner; c += blockDim.x * gridDim.y) {
    float d = dt_bias[c];
    const float* wr = w_up + (long long)c * R;
    for (int j = 0; j < R; ++j) d += wr[j] * mean[j];
    const int h = c / D;
    alpha[(long long)f * inner + c] = __expf(-__expf(a_log[h]) * softplusf_(d));
  }
}

// ---------------------------------------------------------------------------------
// 4. Frame statistics.  K, V FHSD bf16 [F, H, T, D]; beta logits [rows, ld_beta] fp32 with
// row = f*T + s, column beta_col0 + h.  A, B out [F, H, D, D] fp32.  grid (H, F), 256 thr.
// ---------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256) frame_stats_kernel(const __nv_bfloat16* __restrict__ K,
                                                          const __nv_bfloat16* __restrict__ V, int T, int H,
                                                          const float* __restrict__ beta_logits,
                                                          long long ld_beta, int beta_col0,
                                                          float* __restrict__ A, float* __restrict__ Bm) {
  constexpr int CH = 32;        // tokens per chunk
  constexpr int TB = D / 16;    // per-thread block edge: 8 for D=128, 4 for D=64
  __shared__ float sk[CH][D];
  __shared__ float sv[CH][D];
  __shared__ float sb[CH];
  const int h = blockIdx.x, f = blockIdx.y;
  const int ti = threadIdx.x / 16, tj = threadIdx.x % 16;  // 16 x 16 thread grid
  const int i0 = ti * TB, j0 = tj * TB;
  float a[TB][TB], b[TB][TB];
#pragma unroll
  for (int i = 0; i < TB; ++i)
#pragma unroll
    for (int j = 0; j < TB; ++j) a[i][j] = b[i][j] = 0.f;
  const long long base = ((long long)f * H + h) * T * D;
  for (int s0 = 0; s0 < T; s0 += CH) {
    __syncthreads();
    for (int e = threadIdx.x; e < CH * D; e += 256) {
      const int s = e / D, d = e % D;
      const bool in = s0 + s < T;
      sk[s][d] = in ? __bfloat162float(K[base + (long long)(s0 + s) * D + d]) : 0.f;
      sv[s][d] = in ? __bfloat162float(V[base + (long long)(s0 + s) * D + d]) : 0.f;
    }
    if (threadIdx.x < CH) {
      const int s = s0 + threadIdx.x;
      sb[threadIdx.x] = s < T ? sigmoidf_(beta_logits[((long long)f * T + s) * ld_beta + beta_col0 + h]) : 0.f;
    }
    __syncthreads();
    const int n = min(CH, T - s0);
    for (int s = 0; s < n; ++s) {
      const float bt = sb[s];
      float ki[TB], vi[TB], kj[TB];
#pragma unroll
      for (int i = 0; i < TB; ++i) {
        ki[i] = sk[s][i0 + i] * bt;
        vi[i] = sv[s][i0 + i] * bt;
        kj[i] = sk[s][j0 + i];
      }
#pragma unroll
      for (int i = 0; i < TB; ++i)
#pragma unroll
        for (int j = 0; j < TB; ++j) {
          a[i][j] += ki[i] * kj[j];
          b[i][j] += vi[i] * kj[j];
        }
    }
  }
  const long long ob = ((long long)f * H + h) * D * D;
#pragma unroll
  for (int i = 0; i < TB; ++i)
#pragma unroll
    for (int j = 0; j < TB; ++j) {
      A[ob + (long long)(i0 + i) * D + j0 + j] = a[i][j];
      Bm[ob + (long long)(i0 + i) * D + j0 + j] = b[i][j];
    }
}

// ---------------------------------------------------------------------------------
// 5. Delta factor: inv = (I + sym(A))^-1 by in-place Gauss-Jordan elimination without
// pivoting, the matrix held in registers (one TBxTB block per thread of a 16x16 grid).
// For a symmetric matrix the step-k pivot is the ratio of the k-th and (k-1)-th leading
// principal minors, so the first non-positive pivot gives exactly cholesky_ex's info
// (order of the first leading minor that is not positive definite, branch.py:62-71).
// grid (H, F), 256 threads.  info[f, h] = 0 when SPD.
// ---------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256) spd_inverse_kernel(const float* __restrict__ A, int H, float* __restrict__ inv_out,
                                                          int* __restrict__ info,
                                                          __nv_bfloat16* __restrict__ inv_split) {
  constexpr int TB = D / 16;
  // pivot column / row of step k in buffer k & 1: one barrier per step suffices, since a
  // buffer is rewritten two steps later, after every thread has passed the barrier between
  __shared__ __align__(16) float colk[2][D];
  __shared__ __align__(16) float rowk[2][D];
  const int h = blockIdx.x, f = blockIdx.y;
  const long long mb = ((long long)f * H + h) * D * D;
  const int ti = threadIdx.x / 16, tj = threadIdx.x % 16;
  const int r0 = ti * TB, c0 = tj * TB;
  float m[TB][TB];
#pragma unroll
  for (int i = 0; i < TB; ++i)
#pragma unroll
    for (int j = 0; j < TB; ++j) {
      const int r = r0 + i, c = c0 + j;
      m[i][j] = 0.5f * (A[mb + (long long)r * D + c] + A[mb + (long long)c * D + r]) + (r == c ? 1.f : 0.f);
    }
  int bad = 0;
  // k = kb * TB + kr: the block kb is a loop variable, the offset kr is unrolled so every
  // register of m is addressed statically
  for (int kb = 0; kb < 16 && !bad; ++kb) {
#pragma unroll
    for (int kr = 0; kr < TB; ++kr) {
      const int k = kb * TB + kr;
      const int pb = kr & 1;
      if (tj == kb) {
#pragma unroll
        for (int i = 0; i < TB; ++i) colk[pb][r0 + i] = m[i][kr];
      }
      if (ti == kb) {
#pragma unroll
        for (int j = 0; j < TB; ++j) rowk[pb][c0 + j] = m[kr][j];
      }
      __syncthreads();
      const float p = rowk[pb][k];
      if (!(p > 0.f)) {  // uniform: every thread read the same pivot
        bad = k + 1;
        break;
      }
      const float ip = __frcp_rn(p);  // the correctly rounded 1 / p
      float a_i[TB], b_j[TB];
#pragma unroll
      for (int i = 0; i < TB; ++i) a_i[i] = colk[pb][r0 + i] * ip;
#pragma unroll
      for (int j = 0; j < TB; ++j) b_j[j] = rowk[pb][c0 + j];
#pragma unroll
      for (int i = 0; i < TB; ++i) {
        const float2 na = make_float2(-a_i[i], -a_i[i]);
#pragma unroll
        for (int j = 0; j < TB; j += 2) {
          const float2 v = fma2(na, make_float2(b_j[j], b_j[j + 1]), make_float2(m[i][j], m[i][j + 1]));
          m[i][j] = v.x;
          m[i][j + 1] = v.y;
        }
      }
      // row k: a_kj / p ; column k: -a_ik / p ; pivot: 1 / p
      if (ti == kb) {
#pragma unroll
        for (int j = 0; j < TB; ++j) m[kr][j] = b_j[j] * ip;
      }
      if (tj == kb) {
#pragma unroll
        for (int i = 0; i < TB; ++i) m[i][kr] = (r0 + i == k) ? ip : -a_i[i];
      }
    }
  }
  if (threadIdx.x == 0) info[(long long)f * H + h] = bad;
  const float nan = __int_as_float(0x7fc00000);
#pragma unroll
  for (int i = 0; i < TB; ++i)
#pragma unroll
    for (int j = 0; j < TB; ++j) inv_out[mb + (long long)(r0 + i) * D + c0 + j] = bad ? nan : m[i][j];
  if (inv_split) {
    // the same inverse as two bf16 matrices hi + lo (hi = bf16(x), lo = bf16(x - hi)) for the
    // tensor-core scan: hi at inv_split, lo F*H*D*D elements further
    __nv_bfloat16* hi = inv_split + mb;
    __nv_bfloat16* lo = inv_split + (long long)gridDim.y * H * D * D + mb;
#pragma unroll
    for (int i = 0; i < TB; ++i)
#pragma unroll
      for (int j = 0; j < TB; j += 2) {
        const float x0 = bad ? nan : m[i][j], x1 = bad ? nan : m[i][j + 1];
        const __nv_bfloat162 h2 = __floats2bfloat162_rn(x0, x1);
        const float2 hf = __bfloat1622float2(h2);
        *reinterpret_cast<__nv_bfloat162*>(hi + (long long)(r0 + i) * D + c0 + j) = h2;
        *reinterpret_cast<__nv_bfloat162*>(lo + (long long)(r0 + i) * D + c0 + j) =
            __floats2bfloat162_rn(x0 - hf.x, x1 - hf.y);
      }
  }
}

// s0[h] = scale * B[f_text, h] inv[f_text, h] (the text state, branch.py:649-670).
// grid H, 256 threads; each thread computes TB x TB entries.
template <int D>
__global__ void __launch_bounds__(256) text_state_kernel(const float* __restrict__ Bm, const float* __restrict__ inv,
                                                         int H, int text_frame, float scale, float* __restrict__ s0) {
  constexpr int TB = D / 16;
  const int h = blockIdx.x;
  const long long mb = ((long long)text_frame * H + h) * D * D;
  const int r0 = (threadIdx.x / 16) * TB, c0 = (threadIdx.x % 16) * TB;
  float acc[TB][TB] = {};
  for (int k = 0; k < D; ++k) {
    float a[TB], b[TB];
#pragma unroll
    for (int i = 0; i < TB; ++i) a[i] = Bm[mb + (long long)(r0 + i) * D + k];
#pragma unroll
    for (int j = 0; j < TB; ++j) b[j] = inv[mb + (long long)k * D + c0 + j];
#pragma unroll
    for (int i = 0; i < TB; ++i)
#pragma unroll
      for (int j = 0; j < TB; ++j) acc[i][j] += a[i] * b[j];
  }
#pragma unroll
  for (int i = 0; i < TB; ++i)
#pragma unroll
    for (int j = 0; j < TB; ++j) s0[((long long)h * D + r0 + i) * D + c0 + j] = scale * acc[i][j];
}

// The sana_scaled transition factor M = I - A / L (branch.py:163-177; the scan applies the
// alpha scaling and the injection B / sqrt(L) on the fly).  One 32 x 32 tile per CTA
// (32 x 8 threads): M row-major into m_out (optional) and, for the tensor-core scan, M^T as
// bf16 hi / lo halves (its B operand is read K-major, so element [n][k] must hold M[k][n]).
// grid (D/32, D/32, F*H).
__global__ void __launch_bounds__(256) sana_factor_kernel(const float* __restrict__ A, int D, float inv_tokens,
                                                          float* __restrict__ m_out, __nv_bfloat16* __restrict__ split,
                                                          long long lo_offset) {
  __shared__ float tile[32][33];
  const long long mb = (long long)blockIdx.z * D * D;
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int r = r0 + ty + 8 * k, c = c0 + tx;
    const float m = (r == c ? 1.0f : 0.0f) - inv_tokens * A[mb + (long long)r * D + c];
    tile[ty + 8 * k][tx] = m;
    if (m_out) m_out[mb + (long long)r * D + c] = m;
  }
  if (!split) return;
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    // transposed element (n = c0 + ty + 8k, kk = r0 + tx) = M[r0 + tx][c0 + ty + 8k]
    const float x = tile[tx][ty + 8 * k];
    const __nv_bfloat16 hi = __float2bfloat16_rn(x);
    const long long e = mb + (long long)(c0 + ty + 8 * k) * D + r0 + tx;
    split[e] = hi;
    split[lo_offset + e] = __float2bfloat16_rn(x - __bfloat162float(hi));
  }
}

// s0[h] = outer * (inner * B[text_frame, h]): the sana_scaled text state, rounded like the
// reference's two fp32 products (injection, then TEXT_STATE_SCALE; branch.py:649-670).
__global__ void scale_matrix_kernel(const float* __restrict__ Bm, long long n, float inner, float outer,
                                    float* __restrict__ out) {
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x)
    out[e] = outer * (inner * Bm[e]);
}

// ---------------------------------------------------------------------------------
// 6. Bidirectional scan, state rows split across CTAs (the rows of s evolve independently).
// grid (H, 2 directions, D / RB), 256 threads.  states out [F, H, D, D] fp32 (prefix, suffix).
// ---------------------------------------------------------------------------------
template <int D, int RB>
__global__ void __launch_bounds__(256) bidir_scan_kernel(const float* __restrict__ inv, const float* __restrict__ Bm,
                                                         const float* __restrict__ alpha, const float* __restrict__ s0,
                                                         int F, int H, float inj_scale, float* __restrict__ prefix,
                                                         float* __restrict__ suffix) {
  extern __shared__ float sm[];
  float* sinv = sm;             // [D][D]
  float* u = sm + D * D;        // [RB][D]
  const int h = blockIdx.x, dir = blockIdx.y, r0 = blockIdx.z * RB;
  const int tid = threadIdx.x;
  constexpr int OUT = RB * D / 256;  // outputs per thread
  const int r = (tid * OUT) / D, c0 = (tid * OUT) % D;
  float s[OUT];
#pragma unroll
  for (int o = 0; o < OUT; ++o) s[o] = s0 ? s0[((long long)h * D + r0 + r) * D + c0 + o] : 0.f;
  float* dst_all = dir == 0 ? prefix : suffix;
  for (int step = 0; step < F; ++step) {
    const int t = dir == 0 ? step : F - 1 - step;
    const long long mb = ((long long)t * H + h) * D * D;
    __syncthreads();
    for (int e = tid * 4; e < D * D; e += 256 * 4)
      *reinterpret_cast<float4*>(sinv + e) = *reinterpret_cast<const float4*>(inv + mb + e);
    const float* al = alpha + ((long long)t * H + h) * D;
    const float* brow = Bm + mb + (long long)(r0 + r) * D + c0;
    // vdn_solve: u = B + s o alpha, s = u inv;  sana_scaled: u = s o alpha, s = u M + scale B
#pragma unroll
    for (int o = 0; o < OUT; ++o) u[r * D + c0 + o] = inj_scale == 0.f ? brow[o] + s[o] * al[c0 + o] : s[o] * al[c0 + o];
    __syncthreads();
#pragma unroll
    for (int o = 0; o < OUT; ++o) s[o] = 0.f;
    for (int i = 0; i < D; ++i) {
      const float ui = u[r * D + i];
#pragma unroll
      for (int o = 0; o < OUT; ++o) s[o] += ui * sinv[i * D + c0 + o];
    }
    if (inj_scale != 0.f) {
#pragma unroll
      for (int o = 0; o < OUT; ++o) s[o] = fmaf(inj_scale, brow[o], s[o]);
    }
#pragma unroll
    for (int o = 0; o < OUT; ++o) dst_all[mb + (long long)(r0 + r) * D + c0 + o] = s[o];
  }
}

// Head-dim-128 scan: one CTA of 512 threads owns the whole 128 x 128 state of one
// (head, direction), so each frame's inverse crosses L2 once per direction.  Per step:
//   u = B_t + s o alpha_t   (registers -> shared, stored transposed u_t[k][row])
//   s = u (I+A_t)^-1        (register-tiled fp32 GEMM from shared memory: every thread
//                            owns 4 rows x 8 columns, one 16-byte u load and two 16-byte
//                            inverse loads feed 16 paired FMAs per k)
// The next frame's inverse is copied into the second shared buffer by cp.async while
// this frame's product runs, and B_{t+1} is loaded into registers during it.
constexpr int kScanThreads = 512;
constexpr int kScanUPitch = 132;  // u_t row pitch (floats): 16-byte aligned, fewer bank conflicts

__global__ void __launch_bounds__(kScanThreads, 1)
    bidir_scan128_kernel(const float* __restrict__ inv, const float* __restrict__ Bm, const float* __restrict__ alpha,
                         const float* __restrict__ s0, int F, int H, float inj_scale, float* __restrict__ prefix,
                         float* __restrict__ suffix) {
  constexpr int D = 128;
  const bool sana = inj_scale != 0.f;  // u = s o alpha and s = u M + inj_scale B_t
  extern __shared__ __align__(16) float scan_smem[];
  float* sinv = scan_smem;              // [2][D][D]
  float* ut = scan_smem + 2 * D * D;    // [D][kScanUPitch]
  const int h = blockIdx.x, dir = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // warp w: rows 32*(w/4) .. +31, columns 32*(w%4) .. +31; lane: 4 rows x 8 columns
  const int r = 32 * (warp >> 2) + 4 * (lane >> 2);
  const int c = 32 * (warp & 3) + 8 * (lane & 3);
  float* dst_all = dir == 0 ? prefix : suffix;
  auto frame = [&](int step) { return dir == 0 ? step : F - 1 - step; };
  auto issue_inv = [&](int step, int buf) {
    const float* src = inv + ((long long)frame(step) * H + h) * D * D;
    float* dst = sinv + buf * D * D;
#pragma unroll
    for (int i = 0; i < D * D / 4 / kScanThreads; ++i) {
      const int e = (i * kScanThreads + tid) * 4;
      cp_async16(smem_u32(dst + e), src + e);
    }
    cp_async_commit();
  };
  auto load_b = [&](int step, float (&b)[4][8]) {
    const float* src = Bm + ((long long)frame(step) * H + h) * D * D;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 lo = *reinterpret_cast<const float4*>(src + (r + i) * D + c);
      const float4 hi = *reinterpret_cast<const float4*>(src + (r + i) * D + c + 4);
      b[i][0] = lo.x; b[i][1] = lo.y; b[i][2] = lo.z; b[i][3] = lo.w;
      b[i][4] = hi.x; b[i][5] = hi.y; b[i][6] = hi.z; b[i][7] = hi.w;
    }
  };
  float s[4][8], b[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) s[i][j] = s0 ? s0[((long long)h * D + r + i) * D + c + j] : 0.f;
  issue_inv(0, 0);
  load_b(0, b);
  for (int step = 0; step < F; ++step) {
    const int t = frame(step);
    const int buf = step & 1;
    const bool more = step + 1 < F;
    if (more) issue_inv(step + 1, buf ^ 1);
    // u = B_t + s o alpha_t, stored transposed
    const float* al = alpha + ((long long)t * H + h) * D + c;
    const float4 a_lo = *reinterpret_cast<const float4*>(al);
    const float4 a_hi = *reinterpret_cast<const float4*>(al + 4);
    const float av[8] = {a_lo.x, a_lo.y, a_lo.z, a_lo.w, a_hi.x, a_hi.y, a_hi.z, a_hi.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float4 col;
      col.x = fmaf(s[0][j], av[j], sana ? 0.f : b[0][j]);
      col.y = fmaf(s[1][j], av[j], sana ? 0.f : b[1][j]);
      col.z = fmaf(s[2][j], av[j], sana ? 0.f : b[2][j]);
      col.w = fmaf(s[3][j], av[j], sana ? 0.f : b[3][j]);
      *reinterpret_cast<float4*>(ut + (c + j) * kScanUPitch + r) = col;
    }
    if (more) {
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (more && !sana) load_b(step + 1, b);  // in flight during the product
    float2 acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = make_float2(0.f, 0.f);
    const float* iv = sinv + buf * D * D + c;
    const float* uk = ut + r;
#pragma unroll 4
    for (int k = 0; k < D; ++k) {
      const float4 u4 = *reinterpret_cast<const float4*>(uk + k * kScanUPitch);
      const float4 v0 = *reinterpret_cast<const float4*>(iv + k * D);
      const float4 v1 = *reinterpret_cast<const float4*>(iv + k * D + 4);
      const float2 w01 = make_float2(v0.x, v0.y), w23 = make_float2(v0.z, v0.w);
      const float2 w45 = make_float2(v1.x, v1.y), w67 = make_float2(v1.z, v1.w);
      const float uu[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 ui = make_float2(uu[i], uu[i]);
        acc[i][0] = fma2(ui, w01, acc[i][0]);
        acc[i][1] = fma2(ui, w23, acc[i][1]);
        acc[i][2] = fma2(ui, w45, acc[i][2]);
        acc[i][3] = fma2(ui, w67, acc[i][3]);
      }
    }
    float* dst = dst_all + ((long long)t * H + h) * D * D;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[i][2 * j] = sana ? fmaf(inj_scale, b[i][2 * j], acc[i][j].x) : acc[i][j].x;
        s[i][2 * j + 1] = sana ? fmaf(inj_scale, b[i][2 * j + 1], acc[i][j].y) : acc[i][j].y;
      }
      *reinterpret_cast<float4*>(dst + (r + i) * D + c) = make_float4(s[i][0], s[i][1], s[i][2], s[i][3]);
      *reinterpret_cast<float4*>(dst + (r + i) * D + c + 4) = make_float4(s[i][4], s[i][5], s[i][6], s[i][7]);
    }
    if (more && sana) load_b(step + 1, b);  // B_t was needed after the product
    __syncthreads();  // u_t and this inverse buffer are rewritten next step
  }
}

// ---------------------------------------------------------------------------------
// 7. Readout: state (gather + alpha bridge, cast to bf16) -> R = Q S^T -> bf16 ->
// RMSNorm(D) x norm_w -> bf16 -> x output gate -> out rows.
// grid (ceil(T/64), H, F), 256 threads: thread = (4 tokens, D/16 values v = g + 16*vi).
// ---------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256) readout_kernel(
    const __nv_bfloat16* __restrict__ Q, int T, int F, int H, const float* __restrict__ prefix,
    const float* __restrict__ suffix, const float* __restrict__ alpha, const float* __restrict__ s0,
    const int* __restrict__ lo_arr, const int* __restrict__ hi_arr, int use_alpha,
    const float* __restrict__ norm_w, const __nv_bfloat16* __restrict__ gate, long long ld_gate,
    __nv_bfloat16* __restrict__ out, long long ld_out, long long out_row0, int f0, int F_all) {
  constexpr int P = D + 1;
  constexpr int NV = D / 16;
  extern __shared__ float sm[];
  float* st = sm;            // [D][P] state (v, k)
  float* qT = sm + D * P;    // [D][64] q tile, transposed (k, s)
  __shared__ float dec_b[D], dec_a[D];
  const int tile = blockIdx.x, h = blockIdx.y, f = blockIdx.z;
  const int tid = threadIdx.x;
  const int fg = f0 + f;  // clip frame of this call's frame f
  const int raw_lo = lo_arr[fg], raw_hi = hi_arr[fg];
  const int lo = max(raw_lo, 0), hi = min(raw_hi, F_all - 1);
  const bool has_before = raw_lo - 1 >= 0, has_after = raw_hi + 1 < F_all;
  for (int k = tid; k < D; k += 256) {
    float lb = 0.f, la = 0.f;
    if (use_alpha) {
      for (int j = lo; j <= fg; ++j) lb += __logf(fmaxf(alpha[((long long)j * H + h) * D + k], 1e-12f));
      for (int j = fg; j <= hi; ++j) la += __logf(fmaxf(alpha[((long long)j * H + h) * D + k], 1e-12f));
    }
    dec_b[k] = __expf(lb);
    dec_a[k] = __expf(la);
  }
  __syncthreads();
  const float* pb = has_before ? prefix + (((long long)(lo - 1) * H + h) * D * D) : (s0 ? s0 + (long long)h * D * D : nullptr);
  const float* pa = has_after ? suffix + (((long long)(hi + 1) * H + h) * D * D) : (s0 ? s0 + (long long)h * D * D : nullptr);
  for (int e = tid; e < D * D; e += 256) {
    const int v = e / D, k = e % D;
    float val = 0.f;
    if (pb) val += pb[e] * dec_b[k];
    if (pa) val += pa[e] * dec_a[k];
    st[v * P + k] = bf16_round(val);
  }
  const int s_base = tile * 64;
  for (int e = tid; e < 64 * D; e += 256) {
    const int s = e / D, k = e % D;
    qT[k * 64 + s] = (s_base + s < T) ? __bfloat162float(Q[(((long long)f * H + h) * T + s_base + s) * D + k]) : 0.f;
  }
  __syncthreads();
  const int sg = (tid / 16) * 4, g = tid % 16;
  float acc[4][NV];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int vi = 0; vi < NV; ++vi) acc[a][vi] = 0.f;
  for (int k = 0; k < D; ++k) {
    const float4 q4 = *reinterpret_cast<const float4*>(qT + k * 64 + sg);
    float sv[NV];
#pragma unroll
    for (int vi = 0; vi < NV; ++vi) sv[vi] = st[(g + 16 * vi) * P + k];
#pragma unroll
    for (int vi = 0; vi < NV; ++vi) {
      acc[0][vi] += q4.x * sv[vi];
      acc[1][vi] += q4.y * sv[vi];
      acc[2][vi] += q4.z * sv[vi];
      acc[3][vi] += q4.w * sv[vi];
    }
  }
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    float ss = 0.f;
#pragma unroll
    for (int vi = 0; vi < NV; ++vi) {
      acc[a][vi] = bf16_round(acc[a][vi]);
      ss += acc[a][vi] * acc[a][vi];
    }
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss / (float)D + 1e-6f);
    const int tok = s_base + sg + a;
    if (tok < T) {
      const long long local = (long long)f * T + tok;  // row within the branch frames
      const long long row = out_row0 + local;
#pragma unroll
      for (int vi = 0; vi < NV; ++vi) {
        const int v = g + 16 * vi;
        const float nv = bf16_round(acc[a][vi] * inv * norm_w[v]);
        const float gv = __bfloat162float(gate[local * ld_gate + h * D + v]);
        out[row * ld_out + h * D + v] = __float2bfloat16_rn(nv * gv);
      }
    }
  }
}

// fp32 [rows, ld_in] (columns col0..col0+cols) -> bf16 [rows, ld_out]
__global__ void cast_rows_kernel(const float* __restrict__ in, long long ld_in, int col0, int rows, int cols,
                                 __nv_bfloat16* __restrict__ out, long long ld_out) {
  const long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= (long long)rows * cols) return;
  const long long r = e / cols;
  const int c = (int)(e % cols);
  out[r * ld_out + c] = __float2bfloat16_rn(in[r * ld_in + col0 + c]);
}

}  // namespace branch
}  // namespace vdn

using namespace vdn::branch;

extern "C" {

// 1. Depthwise spatial conv (branch.py:469-471).  in rows f*gh*gw + y*gw + x, channels [0, C).
int vdn_spatial_conv(const void* in, long long ld_in, const float* w, int kh, int kw, int F, int gh, int gw, int C,
                     void* out, long long ld_out, void* stream) {
  if (!in || !w || !out || kh <= 0 || kw <= 0 || kh * kw > 49 || (kh % 2) == 0 || (kw % 2) == 0)
    return vdn::kBadArgument;
  if (F <= 0 || gh <= 0 || gw <= 0 || C <= 0) return vdn::kBadArgument;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  const bool paired = kh == 5 && kw == 5 && (C % 2) == 0 && (ld_in % 2) == 0 && (ld_out % 2) == 0 &&
                      (reinterpret_cast<uintptr_t>(in) % 4) == 0 && (reinterpret_cast<uintptr_t>(out) % 4) == 0;
  // tiled path: 16-byte copies of 64-channel slabs
  const long long buf_bytes = (long long)(kConvRows + 4) * (gw + 4) * kConvCh * 2;
  constexpr long long kSmemLimit = 227 * 1024;
  const bool tiled = paired && (C % kConvCh) == 0 && (ld_in % 8) == 0 && vdn::aligned16(in) &&
                     buf_bytes <= kSmemLimit;
  if (tiled) {
    if (!vdn::smem_optin((const void*)spatial_conv5_tiled_kernel, (int)kSmemLimit) ||
        !vdn::func_attr((const void*)spatial_conv5_tiled_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                        cudaSharedmemCarveoutMaxShared))
      return vdn::kLaunchFailed;
    // one buffer per CTA and as many CTAs per SM as fit: some CTAs' copies are in flight
    // while the others compute
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, spatial_conv5_tiled_kernel, kConvThreads,
                                                      (size_t)buf_bytes) != cudaSuccess ||
        per_sm < 1) {
      cudaGetLastError();
      per_sm = 1;
    }
    const long long n_tiles = (long long)(C / kConvCh) * F * ((gh + kConvRows - 1) / kConvRows);
    const int grid = (int)std::min<long long>(n_tiles, (long long)per_sm * vdn::sm_count());
    spatial_conv5_tiled_kernel<<<grid, kConvThreads, buf_bytes, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(in), ld_in, w, F, gh, gw, C, reinterpret_cast<__nv_bfloat16*>(out),
        ld_out);
    vdn::count_launch();
  } else if (paired) {
    dim3 grid((C / 2 + 127) / 128, gh, F);
    spatial_conv5_kernel<<<grid, 128, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(in), ld_in, w, gh, gw, C,
                                              reinterpret_cast<__nv_bfloat16*>(out), ld_out);
    vdn::count_launch();
  } else {
    dim3 grid(gh, F, (C + 255) / 256);
    spatial_conv_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(in), ld_in, w, kh, kw, gh, gw,
                                             C, reinterpret_cast<__nv_bfloat16*>(out), ld_out);
    vdn::count_launch();
  }
  return vdn::launch_status();
}

// 1+2 fused: short conv features of F frames in one pass (branch.py:443-480 + kernels.py:99-129).
// in: raw rows (f*gh + y)*gw + x at pitch ld_in, channel h*D + d (bf16); w_sp [H*D, kh*kw]
// fp32; w_tm [H*D, taps] fp32; out FHSD [F, H, gh*gw, D] bf16.  Same result as
// vdn_spatial_conv followed by vdn_temporal_act.  kUnsupported unless kh = kw = taps = 5
// and D is 64 or 128 (the two-kernel path covers the rest).
int vdn_conv_features(const void* in, long long ld_in, const float* w_sp, int kh, int kw, const float* w_tm, int taps,
                      int F, int gh, int gw, int H, int D, int l2norm, void* out, void* stream) {
  using namespace vdn::branch;
  if (!in || !w_sp || !w_tm || !out || F <= 0 || gh <= 0 || gw <= 0 || H <= 0) return vdn::kBadArgument;
  if (kh != 5 || kw != 5 || taps != 5 || (D != 64 && D != 128)) return vdn::kUnsupported;
  if (!vdn::aligned16(in) || (ld_in % 8) || (reinterpret_cast<uintptr_t>(out) % 4)) return vdn::kMisaligned;
  const int cblocks = (gw + kFeatMaxCols - 1) / kFeatMaxCols;
  const int wc = (gw + cblocks - 1) / cblocks;
  const long long units = (long long)H * ((gh + kFeatRows - 1) / kFeatRows) * cblocks;
  const int grid = (int)std::min<long long>(units, vdn::sm_count());
  auto s = reinterpret_cast<cudaStream_t>(stream);
  const auto* x = reinterpret_cast<const __nv_bfloat16*>(in);
  auto* y = reinterpret_cast<__nv_bfloat16*>(out);
  if (D == 128) {
    const int smem = (int)FeatLayout<128>::bytes(wc);
    if (!vdn::smem_optin((const void*)conv_features_kernel<128>, smem)) return vdn::kLaunchFailed;
    conv_features_kernel<128><<<grid, FeatLayout<128>::kThreads, smem, s>>>(x, ld_in, w_sp, w_tm, F, gh, gw, H, wc,
                                                                            l2norm, y);
  } else {
    const int smem = (int)FeatLayout<64>::bytes(wc);
    if (!vdn::smem_optin((const void*)conv_features_kernel<64>, smem)) return vdn::kLaunchFailed;
    conv_features_kernel<64><<<grid, FeatLayout<64>::kThreads, smem, s>>>(x, ld_in, w_sp, w_tm, F, gh, gw, H, wc,
                                                                          l2norm, y);
  }
  vdn::count_launch();
  return vdn::launch_status();
}

// 2. Temporal 5-tap conv (taps = 5) or none (taps = 0), SiLU, optional L2; FHSD output.
// Replaces kernels.py:99-162 (temporal) and kernels.py:47-51 + the FHSD permute.
int vdn_temporal_act(const void* in, long long ld_in, const float* w, int taps, int F, int T, int H, int D,
                     int l2norm, void* out, void* stream) {
  if (!in || !out || (taps != 0 && taps != 1 && taps != 3 && taps != 5) || (taps && !w)) return vdn::kBadArgument;
  if (D != 64 && D != 128) return vdn::kUnsupported;
  // one D/32-channel vector per lane: 8-byte (D = 128) or 4-byte (D = 64) loads and stores
  const int vec_bytes = D / 16;
  if ((reinterpret_cast<uintptr_t>(out) % vec_bytes) || (reinterpret_cast<uintptr_t>(in) % vec_bytes) ||
      ((ld_in * 2) % vec_bytes))
    return vdn::kMisaligned;
  const long long warps = (long long)T * H;
  const int blocks = (int)((warps * 32 + 255) / 256);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  auto launch = [&](auto kernel) {
    kernel<<<blocks, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(in), ld_in, w, taps, F, T, H, l2norm,
                                  reinterpret_cast<__nv_bfloat16*>(out));
  };
  if (D == 128)
    launch(taps == 5 ? temporal_act_kernel<128, 5> : taps == 3 ? temporal_act_kernel<128, 3> : temporal_act_kernel<128, 1>);
  else
    launch(taps == 5 ? temporal_act_kernel<64, 5> : taps == 3 ? temporal_act_kernel<64, 3> : temporal_act_kernel<64, 1>);
  vdn::count_launch();
  return vdn::launch_status();
}

// 3. alpha gate (branch.py:483-491, frame mean :743-745).  down: [F*T, ld_down] fp32 holding
// x W_down^T (R columns); w_up [H*D, R] fp32; alpha out [F, H, D] fp32.
int vdn_alpha_gate(const float* down, long long ld_down, int F, int T, int R, const float* w_up,
                   const float* dt_bias, const float* a_log, int H, int D, float* alpha, void* stream) {
  if (!down || !w_up || !dt_bias || !a_log || !alpha || F <= 0 || T <= 0 || R <= 0) return vdn::kBadArgument;
  if (R > 4096) return vdn::kUnsupported;
  dim3 grid(F, (H * D + kAlphaThreads - 1) / kAlphaThreads);
  alpha_gate_kernel<<<grid, kAlphaThreads, (R + kAlphaThreads) * sizeof(float),
                      reinterpret_cast<cudaStream_t>(stream)>>>(
      down, ld_down, T, R, w_up, dt_bias, a_log, H, D, alpha);
  vdn::count_launch();
  return vdn::launch_status();
}

// 4. Frame statistics (branch.py:197-243).  K, V FHSD [F, H, T, D] bf16.
int vdn_frame_stats(const void* K, const void* V, int F, int H, int T, int D, const float* beta_logits,
                    long long ld_beta, int beta_col0, float* A, float* B, void* stream) {
  if (!K || !V || !beta_logits || !A || !B) return vdn::kBadArgument;
  dim3 grid(H, F);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (D == 128)
    frame_stats_kernel<128><<<grid, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(K),
                                                 reinterpret_cast<const __nv_bfloat16*>(V), T, H, beta_logits,
                                                 ld_beta, beta_col0, A, B);
  else if (D == 64)
    frame_stats_kernel<64><<<grid, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(K),
                                                reinterpret_cast<const __nv_bfloat16*>(V), T, H, beta_logits,
                                                ld_beta, beta_col0, A, B);
  else
    return vdn::kUnsupported;
  vdn::count_launch();
  return vdn::launch_status();
}

// 5. Delta factor (branch.py:148-160, info semantics of cholesky_ex as in :62-71).
// A, B: [F, H, D, D] fp32.  inv out [F, H, D, D]; info [F, H] int32.  If text_frame >= 0,
// s0 [H, D, D] = text_scale * B[text_frame] inv[text_frame] (branch.py:649-670).
int vdn_delta_factor(const float* A, const float* B, int F, int H, int D, float* inv, int* info, int text_frame,
                     float text_scale, float* s0, void* inv_split, void* stream) {
  if (!A || !inv || !info || (text_frame >= 0 && (!B || !s0))) return vdn::kBadArgument;
  if (text_frame >= F) return vdn::kBadArgument;
  if (inv_split && (D != 128 || (reinterpret_cast<uintptr_t>(inv_split) & 3))) return vdn::kBadArgument;
  dim3 grid(H, F);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  auto* split = reinterpret_cast<__nv_bfloat16*>(inv_split);
  if (D == 128) {
    spd_inverse_kernel<128><<<grid, 256, 0, s>>>(A, H, inv, info, split);
    vdn::count_launch();
    if (text_frame >= 0) {
      text_state_kernel<128><<<H, 256, 0, s>>>(B, inv, H, text_frame, text_scale, s0);
      vdn::count_launch();
    }
  } else if (D == 64) {
    spd_inverse_kernel<64><<<grid, 256, 0, s>>>(A, H, inv, info, nullptr);
    vdn::count_launch();
    if (text_frame >= 0) {
      text_state_kernel<64><<<H, 256, 0, s>>>(B, inv, H, text_frame, text_scale, s0);
      vdn::count_launch();
    }
  } else {
    return vdn::kUnsupported;
  }
  return vdn::launch_status();
}

// 5b. sana_scaled factor (branch.py:163-177): M = I - inv_tokens * A for F frames, row-major
// into M (optional) and transposed as bf16 hi / lo halves into M_split (head_dim 128, optional;
// lo halves F*H*D*D elements after the hi halves, the layout vdn_bidir_scan_tc reads).  If
// text_frame >= 0: s0 = text_scale * (text_inj_scale * B[text_frame]) (branch.py:649-670).
int vdn_sana_factor(const float* A, const float* B, int F, int H, int D, float inv_tokens, float* M, void* M_split,
                    int text_frame, float text_inj_scale, float text_scale, float* s0, void* stream) {
  if (!A || F <= 0 || H <= 0 || (text_frame >= 0 && (!B || !s0)) || text_frame >= F) return vdn::kBadArgument;
  if (D != 64 && D != 128) return vdn::kUnsupported;
  if (M_split && (D != 128 || (reinterpret_cast<uintptr_t>(M_split) & 3))) return vdn::kBadArgument;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (M || M_split) {
    const long long mats = (long long)F * H;
    if (mats > 65535) return vdn::kUnsupported;  // grid z
    sana_factor_kernel<<<dim3(D / 32, D / 32, (unsigned)mats), 256, 0, s>>>(
        A, D, inv_tokens, M, reinterpret_cast<__nv_bfloat16*>(M_split), mats * D * D);
    vdn::count_launch();
  }
  if (text_frame >= 0) {
    const long long n = (long long)H * D * D;
    scale_matrix_kernel<<<(unsigned)((n + 1023) / 1024), 256, 0, s>>>(B + (long long)text_frame * n, n,
                                                                       text_inj_scale, text_scale, s0);
    vdn::count_launch();
  }
  return vdn::launch_status();
}

// 6. Bidirectional scan (branch.py:297-312 with the factor applied on the fly).
// inv, B: [F, H, D, D]; alpha [F, H, D]; s0 [H, D, D] or NULL (zero start).  inj_scale = 0:
// vdn_solve, s_t = (B_t + s_{t-1} o alpha_t) inv_t;  inj_scale > 0: sana_scaled with inv = M,
// s_t = (s_{t-1} o alpha_t) M_t + inj_scale B_t.
int vdn_bidir_scan(const float* inv, const float* B, const float* alpha, const float* s0, int F, int H, int D,
                   float inj_scale, float* prefix, float* suffix, void* stream) {
  if (!inv || !B || !alpha || !prefix || !suffix || inj_scale < 0.f) return vdn::kBadArgument;
  if (!vdn::aligned16(inv)) return vdn::kMisaligned;  // float4 loads of the inverse
  auto s = reinterpret_cast<cudaStream_t>(stream);
  constexpr int RB = 16;
  if (D == 128) {
    // 16-byte vector access to B, alpha, the states and the inverse
    if (!vdn::aligned16(B) || !vdn::aligned16(alpha) || !vdn::aligned16(prefix) || !vdn::aligned16(suffix))
      return vdn::kMisaligned;
    const size_t smem = (size_t)(2 * 128 * 128 + 128 * kScanUPitch) * sizeof(float);
    if (!vdn::smem_optin((const void*)bidir_scan128_kernel, (int)smem)) return vdn::kLaunchFailed;
    bidir_scan128_kernel<<<dim3(H, 2), kScanThreads, smem, s>>>(inv, B, alpha, s0, F, H, inj_scale, prefix,
                                                                 suffix);
    vdn::count_launch();
  } else if (D == 64) {
    const size_t smem = (size_t)(64 * 64 + 2 * RB * 64) * sizeof(float);
    bidir_scan_kernel<64, 2 * RB><<<dim3(H, 2, 64 / (2 * RB)), 256, smem, s>>>(inv, B, alpha, s0, F, H, inj_scale,
                                                                               prefix, suffix);
    vdn::count_launch();
  } else {
    return vdn::kUnsupported;
  }
  return vdn::launch_status();
}

// 7. Readout + epilogue (branch.py:372-396, :494-530, :780).  Q FHSD [F, H, T, D] bf16;
// lo/hi [F] int32 raw window bounds of the branch frames; gate [F*T, ld_gate] bf16 holding
// sigmoid(up(down x) + b) per branch row; out rows out_row0 + f*T + s, columns h*D + v.
int vdn_readout(const void* Q, int F, int H, int T, int D, const float* prefix, const float* suffix,
                const float* alpha, const float* s0, const int* lo, const int* hi, int use_alpha,
                const float* norm_w, const void* gate, long long ld_gate, void* out, long long ld_out,
                long long out_row0, int f0, int F_all, void* stream) {
  if (!Q || !prefix || !suffix || !alpha || !lo || !hi || !norm_w || !gate || !out) return vdn::kBadArgument;
  if (F <= 0 || f0 < 0 || F_all < f0 + F) return vdn::kBadArgument;
  dim3 grid((T + 63) / 64, H, F);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  const size_t smem = (size_t)(D * (D + 1) + D * 64) * sizeof(float);
  if (D == 128) {
    if (!vdn::smem_optin((const void*)readout_kernel<128>, (int)smem)) return vdn::kLaunchFailed;
    readout_kernel<128><<<grid, 256, smem, s>>>(reinterpret_cast<const __nv_bfloat16*>(Q), T, F, H, prefix, suffix,
                                                alpha, s0, lo, hi, use_alpha, norm_w,
                                                reinterpret_cast<const __nv_bfloat16*>(gate), ld_gate,
                                                reinterpret_cast<__nv_bfloat16*>(out), ld_out, out_row0, f0, F_all);
    vdn::count_launch();
  } else if (D == 64) {
    readout_kernel<64><<<grid, 256, smem, s>>>(reinterpret_cast<const __nv_bfloat16*>(Q), T, F, H, prefix, suffix,
                                               alpha, s0, lo, hi, use_alpha, norm_w,
                                               reinterpret_cast<const __nv_bfloat16*>(gate), ld_gate,
                                               reinterpret_cast<__nv_bfloat16*>(out), ld_out, out_row0, f0, F_all);
    vdn::count_launch();
  } else {
    return vdn::kUnsupported;
  }
  return vdn::launch_status();
}

// fp32 -> bf16 copy of a column block (used for the output-gate bottleneck, which the
// reference rounds to the activation dtype: branch.py:755).
int vdn_cast_rows(const float* in, long long ld_in, int col0, int rows, int cols, void* out, long long ld_out,
                  void* stream) {
  if (!in || !out || rows < 0 || cols <= 0) return vdn::kBadArgument;
  const long long n = (long long)rows * cols;
  if (n == 0) return vdn::kOk;
  cast_rows_kernel<<<(unsigned)((n + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      in, ld_in, col0, rows, cols, reinterpret_cast<__nv_bfloat16*>(out), ld_out);
  vdn::count_launch();
  return vdn::launch_status();
}

}  // extern "C"
