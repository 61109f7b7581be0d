// Exact block-sparse window softmax attention for VDN-H3 on sm_100a (tcgen05 + TMA).
//
// Semantics (window.py:277-344): a query row may attend to key row k iff
//     global(q) or global(k) or lo[frame(q)] <= frame(k) <= hi[frame(q)]
//     or (anchor columns and frame(k) in {0, F-1}) or (anchor rows and frame(q) in {0, F-1}),
// softmax over the allowed keys with scale D^-0.5, then the per-token head gate
// sigmoid(x W_g^T + b) (hybrid.py:518-528) is applied and the result is stored in the
// flattened [S, H*D] layout the out-projection reads (softmax_kernels.py:8-9).
//
// B200 design:
//   * persistent CTAs claim (head, 256-row query tile) items from a global queue; the host
//     plan gives each query tile the merged key intervals its rows can see, cut into 128-key
//     tiles at arbitrary row offsets (TMA rows have no alignment rule); only tiles where some
//     row cannot see every key carry a mask flag, and the mask is then rebuilt per element
//     from the frame index (never materialised);
//   * the 256 query rows are two 128-row tiles (a = 0, 1) that share every K/V tile: warp 8
//     streams Q and a 2-stage K/V ring with TMA, warp 9 issues all tcgen05 MMAs (the whole
//     warp runs the issue loop, one elected lane issues), and two softmax warpgroups (warps
//     0-3 for a = 0, 4-7 for a = 1) ping-pong against it; warps 8-11 hand registers to the
//     softmax warpgroups at start-up (setmaxnreg: 80 and 208);
//   * the score MMAs read Q and K from shared memory (8 KB per 64-cycle M128 N128 K16
//     product), the PV MMAs read V (4 KB), and TMA writes 64 KB per K/V tile: 256 KB of
//     shared-memory traffic per 2048 tensor cycles, the shared-memory port's full rate, so
//     the tensor pipe and every barrier operation wait on shared memory when both run;
//   * TMEM (512 columns): S_a in columns [128a, 128a+128), O_a in [256+128a, 384+128a).  The
//     softmax writes P_a as packed bf16 over the first 64 columns of S_a and the PV MMA reads
//     it straight from TMEM (A operand in tensor memory), so shared memory holds only Q and
//     the K/V ring.  The next S_a is issued after PV_a, so the in-order tensor pipe never
//     overwrites P before it is consumed, and S_a's completion implies PV_a's.  P goes to the
//     MMA warp in two parts (keys 0-47, then 48-127), so PV_a starts while the softmax is
//     still on the tile;
//   * online softmax in registers with exp2 in log2 units; the reference maximum moves only
//     when a tile exceeds it by more than 2^8, so O is rescaled rarely (the result is exact),
//     and the exponentials start against the current reference while the tile maximum is
//     still being reduced (a tile is redone when the reference has to move); a quarter of
//     the exponentials run as a paired-fp32 polynomial on the FMA pipe;
//   * the epilogue applies 1/l and the gate and writes bf16 rows.
#include "host_common.h"
#include "sm100.cuh"

namespace vdn {
namespace attn {

constexpr int kThreads = 384;  // 8 softmax warps, 1 TMA warp, 1 MMA warp, 2 warps that only give up registers
// Registers per thread after the start-up reallocation.  The launch holds 168 per thread
// (65,536 / 384, rounded down to a multiple of 8), and each SM sub-partition (16,384
// registers) hosts one warp of each warpgroup: two softmax warps and one of warps 8-11.
// Per sub-partition 2 x 208 + 80 = 496 <= 512 registers per lane; per CTA
// 256 x 208 + 128 x 80 = 63,488 <= 384 x 168 = 64,512.
constexpr int kRegsSoftmax = 208;
constexpr int kRegsIssue = 80;  // warps 8-11: the TMA and MMA warps and two idle warps

template <int N>
__device__ __forceinline__ void reg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void reg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
constexpr int BQ = 128;        // rows per query tile (two per work item)
constexpr int BKV = 128;
constexpr int kStages = 2;
constexpr int kItemRing = 4;

struct Params {
  int S, H, D;
  int vs, ve, F, tpf;
  int anchor_rows, anchor_cols;
  float scale_log2;
  const int* frame_lo;   // [F] first visible key frame (clamped)
  const int* frame_hi;   // [F] last visible key frame (clamped)
  const int* items;      // [n_items] (head << 20) | query tile
  int n_items;
  const int* tile_off;   // [n_qtiles + 1]
  const int* qtile;      // [n_qtiles][2] per 128-row half: (row0 << 8) | rows, rows <= 128 (0: empty
                         // half, row0 still a valid row); null: half a = rows [256 t + 128 a, +128)
  const int* ktile;      // [n_ktiles] (k0 << 9) | (masked << 8) | (valid - 1)
  __nv_bfloat16* out;
  long long ld_out;
  const float* gate_logits;  // [S, ld_gate] fp32 or null
  long long ld_gate;
  int gate_col0;
  const float* gate_bias;    // [H] or null
  int* work_counter;         // zeroed before the launch; items are claimed with atomicAdd
};

// (first row << 8) | rows of half `a` of query tile `qt`: the two halves of a work item may
// come from different places of the sequence (rows with the same visible keys).
__device__ __forceinline__ int q_half(const Params& p, int qt, int a) {
  return p.qtile ? p.qtile[2 * qt + a] : (((qt * 256 + a * 128) << 8) | 128);
}

// Low min(max(n, 0), 32) bits set.
__device__ __forceinline__ uint32_t bits_below(int n) {
  n = min(max(n, 0), 32);
  return n == 32 ? 0xFFFFFFFFu : ((1u << n) - 1u);
}

// Bits [a, b) of a 32-bit word (clamped to the word; empty when b <= a).
__device__ __forceinline__ uint32_t bit_span(int a, int b) { return bits_below(b) & ~bits_below(a); }

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for two values x <= 8 on the FMA/ALU pipes, with the paired fp32 instructions (about
// five instructions per exponential): x = n + f with n = round(x) (added-magic-number
// rounding, t = x + 1.5 * 2^23 holds n in its low bits) and f in [-0.5, 0.5]; 2^f by a cubic
// fitted here for minimum relative error (max 1.0e-4, far below the bf16 rounding P
// receives); 2^n added to the exponent bits as t's bits shifted left by 23 (those of
// 1.5 * 2^23 vanish modulo 2^32).  Inputs below -126 (masked keys are -inf) are clamped to
// 2^-126 instead of 0: the row sum is at least 2^-32 (the key that set the reference has
// weight >= 2^-32), so such weights stay below fp32 resolution in every sum, and no select
// is spent on exact zeros.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  x.x = fmaxf(x.x, -126.0f);
  x.y = fmaxf(x.y, -126.0f);
  const float2 t = add2(x, make_float2(12582912.0f, 12582912.0f));
  const float2 r = add2(t, make_float2(-12582912.0f, -12582912.0f));  // round(x)
  const float2 f = fma2(r, make_float2(-1.0f, -1.0f), x);              // x - round(x) in [-0.5, 0.5]
  float2 q = fma2(make_float2(0.05500844f, 0.05500844f), f, make_float2(0.24220988f, 0.24220988f));
  q = fma2(q, f, make_float2(0.69328284f, 0.69328284f));
  q = fma2(q, f, make_float2(1.0f, 1.0f));
  return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Key pairs (of the eight in a 16-key chunk) whose exponentials run on the FMA pipe: a
// quarter of them, relieving the MUFU unit (16 exponentials per clock per SM, the same rate
// at which the tensor cores consume scores at head_dim 128).
constexpr uint32_t kPolyPairs = 0x22u;

// Row maximum of one 128-key score tile: four independent 3-input max chains.
template <int N>
__device__ __forceinline__ float row_max(const uint32_t (&sr)[N]) {
  float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
  for (int c = 0; c < N; c += 8) {
#pragma unroll
    for (int u = 0; u < 4; ++u) mq[u] = max3(mq[u], __uint_as_float(sr[c + 2 * u]), __uint_as_float(sr[c + 2 * u + 1]));
  }
  return max3(mq[0], mq[1], fmaxf(mq[2], mq[3]));
}


// 32 lanes x 32 bit x 8 columns TMEM store.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

// 32 lanes x 32 bit x 16 columns TMEM store.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// P = 2^(s * scale - m) for the keys of 16-key chunks [C0, C1) of this thread's row, packed
// as bf16 pairs into TMEM over the first columns of the score tile (key 2c in the low half
// of column c) chunk by chunk, so each chunk's scores die as its P leaves; returns the
// chunks' row sum as two partial sums.
template <int C0, int C1, int N>
__device__ __forceinline__ float2 p_chunks(const uint32_t (&sr)[N], float scale, float m, uint32_t s_tmem) {
  const float2 scale2 = make_float2(scale, scale);
  const float2 negm2 = make_float2(-m, -m);
  float2 rs2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
  for (int c0 = 16 * C0; c0 < 16 * C1; c0 += 16) {
    uint32_t pk[8];
#pragma unroll
    for (int c = 0; c < 16; c += 2) {
      const float2 x = fma2(make_float2(__uint_as_float(sr[c0 + c]), __uint_as_float(sr[c0 + c + 1])), scale2, negm2);
      float2 e;
      if ((kPolyPairs >> (c / 2)) & 1u) {
        e = exp2_poly2(x);
      } else {
        e.x = ex2(x.x);
        e.y = ex2(x.y);
      }
      rs2[(c >> 1) & 1] = add2(rs2[(c >> 1) & 1], e);
      pk[c / 2] = pack_bf16(e.x, e.y);
    }
    tmem_st8(s_tmem + c0 / 2, pk);
  }
  return add2(rs2[0], rs2[1]);
}

// The MMAs below take shared-memory descriptors as two 32-bit words.  The low word holds the
// start-address field (bits 0-13, address >> 4) and the leading byte offset, so a constant
// byte offset inside one buffer is a single add of (offset >> 4) to it (smem addresses stay
// below 256 KB: no carry leaves the field); the high word is a per-layout constant.  This keeps
// the issuing thread at a few instructions per MMA while it shares its scheduler with two
// busy softmax warps.
__device__ __forceinline__ uint32_t sdesc_lo(uint32_t saddr, uint32_t lbo) {
  return ((saddr >> 4) & 0x3FFFu) | (((lbo >> 4) & 0x3FFFu) << 16);
}
__host__ __device__ constexpr uint32_t sdesc_hi_sw128(uint32_t sbo) {
  return ((sbo >> 4) & 0x3FFFu) | (1u << 14) | (2u << 29);  // version 1 (bit 46), 128-byte swizzle (bits 61-63)
}

// The MMA warp runs its loop with all 32 lanes (every operand is warp-uniform) and each
// tcgen05.mma / commit below is issued by the lane elect.sync picks: the lowest lane of the
// converged warp, the same thread every time, as a commit must come from the thread that
// issued the MMAs it tracks.  An issue loop confined to one lane by a branch runs at about
// a third of the rate of the 64-cycle M128 N128 K16 products.
// S = Q K^T, both operands from shared memory.
__device__ __forceinline__ void mma_ss(uint32_t d, uint32_t a_lo, uint32_t b_lo, uint32_t hi, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 rx;\n\t.reg .b64 da, db;\n\t"
      "elect.sync rx|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %5, 0;\n\t"
      "mov.b64 da, {%1, %3};\n\t"
      "mov.b64 db, {%2, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %4, p;\n\t}" ::"r"(d),
      "r"(a_lo), "r"(b_lo), "r"(hi), "r"(idesc), "r"(accumulate)
      : "memory");
}

// O += P V with P (A operand) in tensor memory.
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a_tmem, uint32_t b_lo, uint32_t b_hi, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 rx;\n\t.reg .b64 db;\n\t"
      "elect.sync rx|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %5, 0;\n\t"
      "mov.b64 db, {%2, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %4, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate)
      : "memory");
}

// tcgen05.commit from the elected lane (the one that issued the MMAs).
__device__ __forceinline__ void commit_elect(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b32 rx;\n\t"
      "elect.sync rx|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(bar)
      : "memory");
}

// A bounded wait by every lane of a warp; the lanes agree on the outcome, so the warp stays
// converged for the elected issues that follow (a lane that gave up makes all of them stop).
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err, int code) {
  const bool r = mbar_wait_inl(bar, parity, abort_flag, err, code);
  return __all_sync(0xffffffffu, r);
}

template <int D>
struct Layout {
  static constexpr int kQTile = BQ * D * 2;
  static constexpr int kKBytes = BKV * D * 2;
  static constexpr int kVBytes = BKV * D * 2;
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + 2 * kQTile;
  static constexpr int kOffV = kOffK + kStages * kKBytes;
  static constexpr int kOffBar = kOffV + kStages * kVBytes;
  static constexpr int kSmem = kOffBar + 512 + 1024;
};

// P of a tile is handed to the MMA warp in two parts: keys [0, kPSplit) (B_PLO) and the rest
// (B_PHI), so the first PV products run while the softmax finishes the last chunks.  Measured
// at config 1, 40 heads (ms per launch): split 96: 7.33, 64: 7.02, 48: 6.84, 32: 7.08.
constexpr int kPSplit = 48;

enum {
  B_QFULL = 0, B_QEMPTY, B_KFULL0, B_KFULL1, B_VFULL0, B_VFULL1, B_KEMPTY0, B_KEMPTY1, B_VEMPTY0, B_VEMPTY1,
  B_SFULL0, B_SFULL1, B_PLO0, B_PLO1, B_PHI0, B_PHI1, B_ODONE0, B_ODONE1, B_OFREE0, B_OFREE1,
  B_IFULL0, B_IFULL1, B_IFULL2, B_IFULL3, B_IEMPTY0, B_IEMPTY1, B_IEMPTY2, B_IEMPTY3, B_COUNT
};

// 384 threads, one CTA per SM.  The launch gives every thread 168 registers; warps 8-11 hand
// most of theirs back at start-up (setmaxnreg) and the softmax warps take 208.
template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    window_attention_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                            const __grid_constant__ CUtensorMap tv, Params p, int* err) {
  using L = Layout<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + B_COUNT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* item_ring = reinterpret_cast<volatile int*>(tmem_slot + 2);  // [kItemRing]
  auto B = [&](int i) { return smem_u32(&bar[i]); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(B(B_QFULL), 1);
    mbar_init(B(B_QEMPTY), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(B(B_KFULL0 + s), 1);
      mbar_init(B(B_VFULL0 + s), 1);
      mbar_init(B(B_KEMPTY0 + s), 1);
      mbar_init(B(B_VEMPTY0 + s), 1);
      mbar_init(B(B_SFULL0 + s), 1);
      mbar_init(B(B_PLO0 + s), 4);
      mbar_init(B(B_PHI0 + s), 4);
      mbar_init(B(B_ODONE0 + s), 1);
      mbar_init(B(B_OFREE0 + s), 4);
    }
    for (int s = 0; s < kItemRing; ++s) {
      mbar_init(B(B_IFULL0 + s), 1);
      mbar_init(B(B_IEMPTY0 + s), 9);  // the MMA thread and the eight softmax warps
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch(&tq);
    tma_prefetch(&tk);
    tma_prefetch(&tv);
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t sQ = smem_u32(smem + L::kOffQ);
  const uint32_t sK = smem_u32(smem + L::kOffK);
  const uint32_t sV = smem_u32(smem + L::kOffV);
  constexpr int kDBlocks = D / 64;  // 64-element (128 B) column blocks per row

  // Register reallocation, one setmaxnreg instruction per warpgroup: warps 8-11 (TMA, MMA
  // and two idle warps) give registers up at the start, the softmax warpgroups take them.
  // Nothing is given back before the CTA exits: an increase waits until the CTA's pool holds
  // enough registers, and a warp that took back its share early could keep the softmax
  // warps' increase waiting for good.
  if (warp >= 8) {
    reg_dec<kRegsIssue>();
    if (warp == 8) {
      if (lane == 0) {
        // ---------------- TMA producer ----------------
        int g = 0;  // global kv tile counter
        for (int it = 0;; ++it) {
          // Dynamic schedule: fetch the next item from the global queue and hand it to the
          // MMA and softmax warps through a small shared-memory ring (-1 ends the loop).
          const int slot = it % kItemRing;
          if (!mbar_wait_inl(B(B_IEMPTY0 + slot), ((it / kItemRing) & 1) ^ 1, abort_flag, err, kErrWaitProducer)) break;
          const int item = atomicAdd(p.work_counter, 1);
          const int code = item < p.n_items ? p.items[item] : -1;
          item_ring[slot] = code;
          mbar_arrive(B(B_IFULL0 + slot));
          if (code < 0) break;
          const int h = code >> 20, qt = code & 0xFFFFF;
          if (!mbar_wait_inl(B(B_QEMPTY), (it & 1) ^ 1, abort_flag, err, kErrWaitProducer)) break;
          mbar_arrive_expect_tx(B(B_QFULL), 2 * L::kQTile);
          for (int a = 0; a < 2; ++a)
            for (int b = 0; b < kDBlocks; ++b)
              tma_load_2d(sQ + a * L::kQTile + b * (BQ * 128), &tq, B(B_QFULL), h * D + b * 64,
                          q_half(p, qt, a) >> 8);
          const int t0 = p.tile_off[qt], t1 = p.tile_off[qt + 1];
          bool ok = true;
          for (int t = t0; t < t1; ++t, ++g) {
            const int st = g & 1;
            const uint32_t ph = (g >> 1) & 1;
            const int k0 = p.ktile[t] >> 9;
            const uint32_t kb = sK + st * L::kKBytes, vb = sV + st * L::kVBytes;
            if (!mbar_wait_inl(B(B_KEMPTY0 + st), ph ^ 1, abort_flag, err, kErrWaitProducer)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(B(B_KFULL0 + st), L::kKBytes);
            for (int b = 0; b < kDBlocks; ++b)
              tma_load_2d(kb + b * (BKV * 128), &tk, B(B_KFULL0 + st), h * D + b * 64, k0);
            if (!mbar_wait_inl(B(B_VEMPTY0 + st), ph ^ 1, abort_flag, err, kErrWaitProducer)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(B(B_VFULL0 + st), L::kVBytes);
            for (int b = 0; b < kDBlocks; ++b)
              tma_load_2d(vb + b * (BKV * 128), &tv, B(B_VFULL0 + st), h * D + b * 64, k0);
          }
          if (!ok) break;
        }
      }
    } else if (warp == 9) {
      {
        // ---------------- MMA issuer ----------------
        constexpr uint32_t idesc_s = make_idesc(1, 1, 1, 0, 0, BQ, BKV);
        constexpr uint32_t idesc_o = make_idesc(1, 1, 1, 0, 1, BQ, D);
        constexpr uint32_t hi_k = sdesc_hi_sw128(1024);  // K-major Q / K, and MN-major V: SBO 1024
        const uint32_t q_lo = sdesc_lo(sQ, 16), k_lo = sdesc_lo(sK, 16), v_lo = sdesc_lo(sV, BKV * 128);
        auto issue_s = [&](int a, int st) {
          const uint32_t qa = q_lo + a * (L::kQTile >> 4), kb = k_lo + st * (L::kKBytes >> 4);
  #pragma unroll
          for (int s = 0; s < D / 16; ++s) {
            const uint32_t off = ((s >> 2) * (BQ * 128) + (s & 3) * 32) >> 4;
            mma_ss(tmem_base + a * 128, qa + off, kb + off, hi_k, idesc_s, s > 0 ? 1u : 0u);
          }
          commit_elect(B(B_SFULL0 + a));
        };
        int g = 0;
        int it = 0;
        bool ok = true;
        for (; ok; ++it) {
          const int slot = it % kItemRing;
          if (!warp_wait(B(B_IFULL0 + slot), (it / kItemRing) & 1, abort_flag, err, kErrWaitMma)) break;
          const int code = item_ring[slot];
          if (lane == 0) mbar_arrive(B(B_IEMPTY0 + slot));
          if (code < 0) break;
          const int qt = code & 0xFFFFF;
          const int n = p.tile_off[qt + 1] - p.tile_off[qt];
          if (!warp_wait(B(B_QFULL), it & 1, abort_flag, err, kErrWaitMma) ||
              !warp_wait(B(B_KFULL0 + (g & 1)), (g >> 1) & 1, abort_flag, err, kErrWaitMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(0, g & 1);
          issue_s(1, g & 1);
          commit_elect(B(B_KEMPTY0 + (g & 1)));
          if (n == 1) commit_elect(B(B_QEMPTY));
          for (int j = 0; j < n && ok; ++j) {
            const int gj = g + j, st = gj & 1;
            const uint32_t ph = (gj >> 1) & 1;
            for (int a = 0; a < 2; ++a) {
              if (!warp_wait(B(B_PLO0 + a), gj & 1, abort_flag, err, kErrWaitMma) ||
                  (j == 0 && !warp_wait(B(B_OFREE0 + a), (it & 1) ^ 1, abort_flag, err, kErrWaitMma)) ||
                  (a == 0 && !warp_wait(B(B_VFULL0 + st), ph, abort_flag, err, kErrWaitMma))) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t vb = v_lo + st * (L::kVBytes >> 4);
  #pragma unroll
              for (int s = 0; s < kPSplit / 16; ++s)
                mma_ts(tmem_base + 256 + a * 128, tmem_base + a * 128 + s * 8, vb + s * (2048 >> 4), hi_k, idesc_o,
                       (j > 0 || s > 0) ? 1u : 0u);
              if (!warp_wait(B(B_PHI0 + a), gj & 1, abort_flag, err, kErrWaitMma)) {
                ok = false;
                break;
              }
              tc_fence_after();
  #pragma unroll
              for (int s = kPSplit / 16; s < BKV / 16; ++s)
                mma_ts(tmem_base + 256 + a * 128, tmem_base + a * 128 + s * 8, vb + s * (2048 >> 4), hi_k, idesc_o, 1u);
              if (a == 1) commit_elect(B(B_VEMPTY0 + st));
              if (j == n - 1) commit_elect(B(B_ODONE0 + a));
              if (j + 1 < n) {
                const int g1 = gj + 1, st1 = g1 & 1;
                if (a == 0 && !warp_wait(B(B_KFULL0 + st1), (g1 >> 1) & 1, abort_flag, err, kErrWaitMma)) {
                  ok = false;
                  break;
                }
                tc_fence_after();
                issue_s(a, st1);
                if (a == 1) {
                  commit_elect(B(B_KEMPTY0 + st1));
                  if (j + 1 == n - 1) commit_elect(B(B_QEMPTY));
                }
              }
            }
          }
          g += n;
        }
      }
    }
  } else {
    reg_inc<kRegsSoftmax>();
    // ---------------- softmax / correction / epilogue: warpgroup a = warp / 4 ----------------
    const int a = warp >> 2;
    const int row_in_tile = (warp & 3) * 32 + lane;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t s_tmem = tmem_base + lane_base + a * 128;
    const uint32_t o_tmem = tmem_base + lane_base + 256 + a * 128;
    int g = 0;
    int it = 0;
    bool ok = true;
    for (; ok; ++it) {
      const int slot = it % kItemRing;
      if (!mbar_wait_inl(B(B_IFULL0 + slot), (it / kItemRing) & 1, abort_flag, err, kErrWaitEpilogue)) break;
      const int code = item_ring[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(B(B_IEMPTY0 + slot));
      if (code < 0) break;
      const int h = code >> 20, qt = code & 0xFFFFF;
      const int t0 = p.tile_off[qt], n = p.tile_off[qt + 1] - t0;
      const int qinfo = q_half(p, qt, a);
      const int qrow = (qinfo >> 8) + row_in_tile;
      // rows past the half's count belong to another tile (or lie past S): computed, not stored
      const bool row_valid = row_in_tile < (qinfo & 0xFF) && qrow < p.S;
      // Per-row visibility (window.py:327-344): a windowed row cannot see the video keys in
      // [x0, x1) and [x2, x3) = [first non-anchor key, window start) and [window end, first
      // key of the last anchor frame); rows that see every key get two empty spans.
      int x0 = 0, x1 = 0, x2 = 0, x3 = 0;
      if (qrow >= p.vs && qrow < p.ve) {
        const int f = (qrow - p.vs) / p.tpf;
        if (!(p.anchor_rows && (f == 0 || f == p.F - 1))) {
          x0 = p.anchor_cols ? p.vs + p.tpf : p.vs;
          x1 = p.vs + p.frame_lo[f] * p.tpf;
          x2 = p.vs + (p.frame_hi[f] + 1) * p.tpf;
          x3 = p.anchor_cols ? p.ve - p.tpf : p.ve;
        }
      }
      float m_run = -INFINITY, l_run = 0.f;
      int info_next = p.ktile[t0];
      for (int j = 0; j < n; ++j) {
        const int gj = g + j;
        const int info = info_next;
        if (j + 1 < n) info_next = p.ktile[t0 + j + 1];  // prefetch the next tile descriptor
        if (!mbar_wait_inl(B(B_SFULL0 + a), gj & 1, abort_flag, err, kErrWaitEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[BKV];  // raw scores of this row (fp32 bits)
        const int k0 = info >> 9;
        const int valid = (info & 0xFF) + 1;
        const bool masked = (info >> 8) & 1;
        {
#pragma unroll
          for (int c = 0; c < BKV / 32; ++c)
            tmem_ld32(s_tmem + c * 32, *reinterpret_cast<uint32_t(*)[32]>(sr + c * 32));
          tmem_ld_wait();
          if (masked || valid < BKV) {
            // visible keys of this row as four 32-key bit words, then one test + select per key
            uint32_t vis[BKV / 32];
#pragma unroll
            for (int w = 0; w < BKV / 32; ++w) {
              const int base = k0 + 32 * w;
              uint32_t m = bits_below(valid - 32 * w);
              if (masked) m &= ~(bit_span(x0 - base, x1 - base) | bit_span(x2 - base, x3 - base));
              vis[w] = m;
            }
#pragma unroll
            for (int c = 0; c < BKV; ++c)
              if (!((vis[c >> 5] >> (c & 31)) & 1u)) sr[c] = __float_as_uint(-INFINITY);
          }
        }
        // The reference max m of a row moves only when a tile's max exceeds it by more than
        // 2^8 (in log2 units), so exponents stay <= 8 and O is rescaled rarely; the result is
        // exact.  The exponentials therefore start against the current reference before the
        // tile max is known (the max chains overlap them), and the tile is redone from the
        // scores still in registers only when the reference has to move.  A row's first tile
        // speculates on m = 0 and keeps it when its max lies within [-32, 8] (the row sum
        // then stays >= 2^-32).
        const float mt = row_max(sr);
        const bool first = (m_run == -INFINITY);
        const float m_spec = first ? 0.f : m_run;
        const float2 lo = p_chunks<0, kPSplit / 16>(sr, p.scale_log2, m_spec, s_tmem);
        const float mts = mt * p.scale_log2;
        const bool grow = first ? (mts > 8.0f || mts < -32.0f) : (mts > m_run + 8.0f);
        if (!__any_sync(0xffffffffu, grow)) {
          // keys [0, kPSplit) are final: the first PV products start while the rest is computed
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(B(B_PLO0 + a));
          const float2 hi = p_chunks<kPSplit / 16, BKV / 16>(sr, p.scale_log2, m_spec, s_tmem);
          const float2 rsum = add2(lo, hi);
          l_run += rsum.x + rsum.y;
          m_run = m_spec;
        } else {
          // some row of this warp moves its reference: redo the tile (rows that do not move
          // recompute the same values), then rescale O
          const float m_new = grow ? mts : m_spec;
          const float m_use = (m_new == -INFINITY) ? 0.f : m_new;  // a fully masked tile keeps 0
          const float corr = grow ? ex2(m_spec - m_use) : 1.0f;  // O and l are relative to m_spec
          tmem_st_wait();  // the speculative stores land before they are overwritten
          const float2 rsum = p_chunks<0, BKV / 16>(sr, p.scale_log2, m_use, s_tmem);
          // O_a is stable here: S_j(a) completed, so PV_{j-1}(a) (issued before it) did too;
          // and PV_j(a) is not issued before this warpgroup signals P_j(a) below.
          if (j > 0) {
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
              uint32_t o[32];
              tmem_ld32(o_tmem + c * 32, o);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
              tmem_st32(o_tmem + c * 32, o);
            }
          }
          l_run = l_run * corr + (rsum.x + rsum.y);
          m_run = m_new;  // stays -inf while every key seen so far was masked
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(B(B_PLO0 + a));
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(B(B_PHI0 + a));
      }
      if (!ok) break;
      g += n;
      // Epilogue: wait for the last PV of this tile, normalise, gate, store.
      if (!mbar_wait_inl(B(B_ODONE0 + a), it & 1, abort_flag, err, kErrWaitEpilogue)) break;
      tc_fence_after();
      float gate = 1.f;
      if (p.gate_logits && row_valid) {
        float z = p.gate_logits[(long long)qrow * p.ld_gate + p.gate_col0 + h];
        if (p.gate_bias) z += p.gate_bias[h];
        gate = 1.f / (1.f + __expf(-z));
      }
      const float inv_l = (l_run > 0.f) ? gate / l_run : 0.f;
      __nv_bfloat16* dst = p.out + (long long)qrow * p.ld_out + h * D;
      // O in 32-column chunks (keeps 32 values live); the accumulator is released after the last
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(o_tmem + c * 32, r);
        tmem_ld_wait();
        if (c == D / 32 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(B(B_OFREE0 + a));
        }
        if (row_valid) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 v;
            v.x = pack_bf16(__uint_as_float(r[i]) * inv_l, __uint_as_float(r[i + 1]) * inv_l);
            v.y = pack_bf16(__uint_as_float(r[i + 2]) * inv_l, __uint_as_float(r[i + 3]) * inv_l);
            v.z = pack_bf16(__uint_as_float(r[i + 4]) * inv_l, __uint_as_float(r[i + 5]) * inv_l);
            v.w = pack_bf16(__uint_as_float(r[i + 6]) * inv_l, __uint_as_float(r[i + 7]) * inv_l);
            *reinterpret_cast<uint4*>(dst + c * 32 + i) = v;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag) abort_drain();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

template <int D>
int launch(const void* q, long long ld_q, const void* k, long long ld_k, const void* v, long long ld_v, Params p,
           int* err, cudaStream_t stream) {
  CUtensorMap tq, tk, tv;
  const uint64_t width = (uint64_t)p.H * D;
  int rc = make_tmap_2d(&tq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, width, (uint64_t)p.S, (uint64_t)ld_q, 64, 128);
  if (rc) return rc;
  rc = make_tmap_2d(&tk, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, width, (uint64_t)p.S, (uint64_t)ld_k, 64, 128);
  if (rc) return rc;
  rc = make_tmap_2d(&tv, v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, width, (uint64_t)p.S, (uint64_t)ld_v, 64, 128);
  if (rc) return rc;
  if (!smem_optin((const void*)window_attention_kernel<D>, Layout<D>::kSmem)) return kLaunchFailed;
  const int grid = p.n_items < sm_count() ? p.n_items : sm_count();
  if (grid <= 0) return kOk;
  window_attention_kernel<D><<<grid, kThreads, Layout<D>::kSmem, stream>>>(tq, tk, tv, p, err);
  vdn::count_launch();
  return launch_status();
}

}  // namespace attn
}  // namespace vdn

extern "C" {

// Window softmax attention with the fused per-token head gate.
//   q, k, v  [S, H*D] bf16 row-major views with row pitches ld_q / ld_k / ld_v (elements);
//            q and k already RMS-normalised (hybrid.py:271-273)
//   out      [S, ld_out] bf16: gated output at columns h*D
//   frame_lo / frame_hi [F] int32 device arrays: clamped visible key-frame range per frame
//   items / tile_off / qtile / ktile: the block-sparse plan built by the host package;
//            qtile [n_qtiles][2] = per 128-row half (first row << 8) | rows, rows <= 128 (0: an
//            empty half whose first row is still a valid row), or null for query tile t =
//            rows [256 t, 256 t + 256)
//   gate_logits [S, ld_gate] fp32 (column gate_col0 + h) and gate_bias [H]: optional
//   work_counter: one device int, zeroed here on the stream; launches that share it must not overlap
// Replaces window.py:277-313 (window_softmax_grouped) + hybrid.py:518-528.
int vdn_window_attention(const void* q, long long ld_q, const void* k, long long ld_k, const void* v, long long ld_v,
                         int S, int H, int D, int video_start, int video_end, int num_frames, int tokens_per_frame,
                         int anchor_rows, int anchor_cols, float scale, const int* frame_lo, const int* frame_hi,
                         const int* items, int n_items, const int* tile_off, const int* qtile, const int* ktile,
                         void* out,
                         long long ld_out, const float* gate_logits, long long ld_gate, int gate_col0,
                         const float* gate_bias, int* work_counter, int* dev_err, void* stream) {
  if (!q || !k || !v || !out || !items || !tile_off || !ktile || !frame_lo || !frame_hi || !work_counter)
    return vdn::kBadArgument;
  if (D != 64 && D != 128) return vdn::kUnsupported;
  if (S <= 0 || H <= 0 || H >= 2048 || num_frames <= 0 || tokens_per_frame <= 0) return vdn::kBadArgument;
  if (S >= (1 << 22)) return vdn::kUnsupported;
  if ((ld_out * 2) % 16 || !vdn::aligned16(out)) return vdn::kMisaligned;  // 16-byte output vectors
  vdn::attn::Params p{};
  p.S = S;
  p.H = H;
  p.D = D;
  p.vs = video_start;
  p.ve = video_end;
  p.F = num_frames;
  p.tpf = tokens_per_frame;
  p.anchor_rows = anchor_rows;
  p.anchor_cols = anchor_cols;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.frame_lo = frame_lo;
  p.frame_hi = frame_hi;
  p.items = items;
  p.n_items = n_items;
  p.tile_off = tile_off;
  p.qtile = qtile;
  p.ktile = ktile;
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.ld_out = ld_out;
  p.gate_logits = gate_logits;
  p.ld_gate = ld_gate;
  p.gate_col0 = gate_col0;
  p.gate_bias = gate_bias;
  p.work_counter = work_counter;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaMemsetAsync(work_counter, 0, sizeof(int), s);
  return D == 128 ? vdn::attn::launch<128>(q, ld_q, k, ld_k, v, ld_v, p, dev_err, s)
                  : vdn::attn::launch<64>(q, ld_q, k, ld_k, v, ld_v, p, dev_err, s);
}

}  // extern "C"
