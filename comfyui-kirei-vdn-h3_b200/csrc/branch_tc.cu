// Tensor-core (tcgen05) kernels of the VDA branch for head_dim 128.
//
//   vdn_frame_stats_tc   A = (beta K)^T K and B = (beta V)^T K per frame and head
//                        (branch.py:197-243): both operands MN-major straight from the FHSD
//                        feature tiles, accumulated over 128-token chunks in TMEM.
//   vdn_readout_tc       gather + alpha bridge into a bf16 state tile (branch.py:372-396), then
//                        R = Q S^T and G = bf16(x W_og_down^T) W_og_up^T on the tensor cores
//                        (branch.py:780, :754-758) and the RMSNorm(D) x sigmoid(G + b) epilogue
//                        (branch.py:494-530) from TMEM: the output-gate up-projection never
//                        touches HBM.
// Both kernels are warp-specialised pipelines (TMA producer, MMA issuer, worker warps,
// double-buffered TMEM accumulators), described above each kernel.
#include "host_common.h"
#include "sm100.cuh"

namespace vdn {
namespace branch_tc {

constexpr int D = 128;
constexpr int kRows = 128;                 // tokens per chunk / tile
constexpr int kTile = kRows * D * 2;       // 32 KB bf16 tile (two 64-column swizzle blocks)
constexpr int kBlk = kRows * 128;          // 16 KB: one 64-column block

__device__ __forceinline__ float sigm(float x) { return 1.0f / (1.0f + __expf(-x)); }

// ------------------------------------------------------------------------------- statistics
// Warp-specialised pipeline (320 threads):
//   warp 0      TMA producer: K and V chunks (128 tokens x 128 features each) of the CTA's
//               (frame, head) units into a 2-stage ring;
//   warps 2-5   scalers (thread = token row): beta = sigmoid(logit) (0 past the frame end),
//               write beta*K into one of two beta-K buffers and scale V in place;
//   warp 1      MMA issuer: A += (beta K)^T K and B += (beta V)^T K (both operands MN-major,
//               straight from the feature tiles) into one of two TMEM accumulator pairs;
//   warps 6-9   epilogue (TMEM lane = feature row): A and B rows of the finished unit to HBM
//               while the next unit accumulates in the other pair.
// smem: 2 x (K, V) + 2 x beta-K = 6 x 32 KB.
struct StatsSmem {
  static constexpr int kKV = 0, kBK = 4 * kTile, kBar = 6 * kTile;
  static constexpr int kBytes = kBar + 256 + 1024;
};
constexpr int kStatsThreads = 320;

__global__ void __launch_bounds__(kStatsThreads, 1)
    frame_stats_tc_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv, int F, int H,
                          int T, const float* __restrict__ beta_logits, long long ld_beta, int beta_col0,
                          float* __restrict__ A, float* __restrict__ Bm, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + StatsSmem::kBar);
  uint64_t* kv_full = bar;       // [2] TMA bytes
  uint64_t* kv_empty = bar + 2;  // [2] MMA commit
  uint64_t* bk_full = bar + 4;   // [2] 4 scaler warps
  uint64_t* bk_empty = bar + 6;  // [2] MMA commit
  uint64_t* acc_full = bar + 8;  // [2] MMA commit
  uint64_t* acc_empty = bar + 10;  // [2] 4 epilogue warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < 12; ++i) mbar_init(smem_u32(&bar[i]), (i == 4 || i == 5 || i == 10 || i == 11) ? 4 : 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch(&tk);
    tma_prefetch(&tv);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sKV = smem_u32(smem + StatsSmem::kKV), sBK = smem_u32(smem + StatsSmem::kBK);
  const int units = F * H;
  const int u0 = (int)((long long)blockIdx.x * units / gridDim.x);
  const int u1 = (int)((long long)(blockIdx.x + 1) * units / gridDim.x);
  const int nch = (T + kRows - 1) / kRows;
  // stage st: K at sKV + st * 2 * kTile, V right after it

  if (warp == 0) {
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int unit = u0; unit < u1 && ok; ++unit) {
        for (int c = 0; c < nch; ++c, ++g) {
          const int st = g & 1;
          if (!mbar_wait(smem_u32(&kv_empty[st]), ((g >> 1) & 1) ^ 1, abort_flag, err, kErrWaitProducer)) {
            ok = false;
            break;
          }
          const int row0 = unit * T + c * kRows;  // FHSD rows: (f * H + h) * T + s
          const uint32_t fb = smem_u32(&kv_full[st]);
          const uint32_t kb = sKV + st * 2 * kTile, vb = kb + kTile;
          mbar_arrive_expect_tx(fb, 2 * kTile);
          for (int b = 0; b < 2; ++b) {
            tma_load_2d(kb + b * kBlk, &tk, fb, b * 64, row0);
            tma_load_2d(vb + b * kBlk, &tv, fb, b * 64, row0);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(1, 1, 1, 1, 1, 128, 128);  // both operands MN-major
      int g = 0, acc = 0;
      uint32_t acc_ph = 0;
      bool ok = true;
      for (int unit = u0; unit < u1 && ok; ++unit) {
        if (!mbar_wait(smem_u32(&acc_empty[acc]), acc_ph ^ 1, abort_flag, err, kErrWaitMma)) break;
        const uint32_t d = tmem + acc * 256;
        for (int c = 0; c < nch; ++c, ++g) {
          const int st = g & 1;
          if (!mbar_wait(smem_u32(&bk_full[st]), (g >> 1) & 1, abort_flag, err, kErrWaitMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t kb = sKV + st * 2 * kTile, vb = kb + kTile, bkb = sBK + st * kTile;
#pragma unroll
          for (int k = 0; k < kRows / 16; ++k) {
            const uint32_t off = k * 2048;  // 16 tokens = two 8-row swizzle groups
            const uint64_t bdesc = make_sdesc(kb + off, kBlk, 1024);
            mma_f16(d, make_sdesc(bkb + off, kBlk, 1024), bdesc, idesc, (c > 0 || k > 0) ? 1u : 0u);
            mma_f16(d + 128, make_sdesc(vb + off, kBlk, 1024), bdesc, idesc, (c > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(smem_u32(&kv_empty[st]));
          tc_commit(smem_u32(&bk_empty[st]));
          if (c == nch - 1) tc_commit(smem_u32(&acc_full[acc]));
        }
        if (++acc == 2) {
          acc = 0;
          acc_ph ^= 1;
        }
      }
    }
  } else if (warp < 6) {
    // scalers: thread = token row of the chunk
    const int r = tid - 64;
    int g = 0;
    bool ok = true;
    // this thread's token logit of a chunk (0 for rows past the frame, which read nothing);
    // the next chunk's is loaded one chunk ahead, so its latency hides behind the waits
    auto logit_of = [&](int unit, int c) -> float {
      const int s = c * kRows + r;
      if (s >= T) return 0.f;
      return beta_logits[((long long)(unit / H) * T + s) * ld_beta + beta_col0 + unit % H];
    };
    float logit_next = u0 < u1 ? logit_of(u0, 0) : 0.f;
    for (int unit = u0; unit < u1 && ok; ++unit) {
      for (int c = 0; c < nch; ++c, ++g) {
        const int st = g & 1;
        const float logit = logit_next;
        if (c + 1 < nch)
          logit_next = logit_of(unit, c + 1);
        else if (unit + 1 < u1)
          logit_next = logit_of(unit + 1, 0);
        // K/V of this chunk landed, and the MMA that read this beta-K buffer two chunks ago is done
        const bool okw = __all_sync(0xffffffffu,
                                    mbar_wait(smem_u32(&kv_full[st]), (g >> 1) & 1, abort_flag, err, kErrWaitOther) &&
                                        mbar_wait(smem_u32(&bk_empty[st]), ((g >> 1) & 1) ^ 1, abort_flag, err,
                                                  kErrWaitOther));
        if (!okw) {
          ok = false;
          break;
        }
        const int s = c * kRows + r;
        uint8_t* kt = smem + StatsSmem::kKV + st * 2 * kTile;
        uint8_t* vt = kt + kTile;
        uint8_t* bk = smem + StatsSmem::kBK + st * kTile;
        // A row past the frame holds the next unit's tokens: it is zeroed in all three operand
        // tiles (a zero beta alone would still carry a non-finite token of the next unit into
        // this unit's sums as 0 * inf), so each frame's statistics see only its own tokens.
        const bool past = s >= T;
        const float beta = past ? 0.f : sigm(logit);
        const __nv_bfloat162 b2 = __floats2bfloat162_rn(beta, beta);
        for (int b = 0; b < 2; ++b) {
          const uint32_t off = b * kBlk + r * 128;
          uint4* srck = reinterpret_cast<uint4*>(kt + off);
          uint4* vv = reinterpret_cast<uint4*>(vt + off);
          uint4* dk = reinterpret_cast<uint4*>(bk + off);
          // the scale is the same for the whole row, so any chunk order works: start each
          // row at a different 16-byte chunk so the eight rows of a quarter-warp hit
          // different banks
#pragma unroll
          for (int i0 = 0; i0 < 8; ++i0) {
            const int i = i0 ^ (r & 7);
            uint4 k4 = srck[i], v4 = vv[i];
            if (past) {
              k4 = make_uint4(0u, 0u, 0u, 0u);
              v4 = k4;
              srck[i] = k4;
            }
            __nv_bfloat162* kp = reinterpret_cast<__nv_bfloat162*>(&k4);
            __nv_bfloat162* vp = reinterpret_cast<__nv_bfloat162*>(&v4);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              kp[e] = __hmul2(kp[e], b2);
              vp[e] = __hmul2(vp[e], b2);
            }
            dk[i] = k4;
            vv[i] = v4;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bk_full[st]));
      }
    }
  } else {
    // epilogue: row i of A and of B from TMEM lane i (quadrant = warp % 4)
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    int acc = 0;
    uint32_t acc_ph = 0;
    for (int unit = u0; unit < u1; ++unit) {
      if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&acc_full[acc]), acc_ph, abort_flag, err, kErrWaitEpilogue)))
        break;
      tc_fence_after();
      const long long ob = ((long long)unit * D + row) * D;
      for (int m = 0; m < 2; ++m) {
        float* dst = (m == 0 ? A : Bm) + ob;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_base + acc * 256 + m * 128 + c * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4*>(dst + c * 32 + i) =
                make_float4(__uint_as_float(v[i]), __uint_as_float(v[i + 1]), __uint_as_float(v[i + 2]),
                            __uint_as_float(v[i + 3]));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&acc_empty[acc]));
      if (++acc == 2) {
        acc = 0;
        acc_ph ^= 1;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) abort_drain();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------------- readout
// Warp-specialised and pipelined (256 threads):
//   warp 0      TMA producer: the output-gate up rows of the current head (once per head,
//               the CTA walks its units head-major), and per 128-token tile the Q tile and
//               the og-down tile into one of two stages;
//   warp 1      MMA issuer: R = Q S^T and G = og_down W_up^T into one of two TMEM
//               accumulator pairs (2 x 256 columns), so tile i+1 is multiplied while the
//               epilogue drains tile i;
//   warps 2-3   state builders: gather + alpha bridge of the NEXT unit's bf16 state into
//               the second state buffer while the current unit's tiles run;
//   warps 4-11  epilogue (TMEM lane = token row, two warps per lane quadrant, one per
//               64-column half): bf16(R) -> RMSNorm x norm_w -> bf16 -> x sigmoid(G + b)
//               -> 16-byte stores.
// smem: 2 state buffers, W_up, 2 stages x (Q, og-down) = 7 x 32 KB.
struct ReadoutSmem {
  static constexpr int kS = 0, kW = 2 * kTile, kQG = 3 * kTile, kBar = 7 * kTile;
  static constexpr int kSsq = kBar + 256;               // epilogue partial sums [2 acc][2 halves][128 rows]
  static constexpr int kBytes = kSsq + 2 * 2 * 128 * 4;  // 231,680 B: no room for alignment slack
};
constexpr int kReadoutThreads = 384;  // 12 warps: producer, MMA, 2 state builders, 8 epilogue

__global__ void __launch_bounds__(kReadoutThreads, 1)
    readout_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tg,
                      const __grid_constant__ CUtensorMap tw, int F, int H, int T, const float* __restrict__ prefix,
                      const float* __restrict__ suffix, const float* __restrict__ alpha, const float* __restrict__ s0,
                      const int* __restrict__ lo_arr, const int* __restrict__ hi_arr, int use_alpha,
                      const float* __restrict__ norm_w, const float* __restrict__ og_bias,
                      __nv_bfloat16* __restrict__ out, long long ld_out, long long out_row0, int f0, int F_all,
                      int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // The layout uses the whole 227 KB, so the dynamic window must start 1024-aligned (it
  // does when the kernel has no static shared memory); otherwise report and leave.
  if (smem_u32(smem_raw) & 1023) {
    if (threadIdx.x == 0) atomicExch(err, kErrWaitOther);
    return;
  }
  uint8_t* smem = smem_raw;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + ReadoutSmem::kBar);
  uint64_t* qg_full = bar;        // [2]
  uint64_t* qg_empty = bar + 2;   // [2]
  uint64_t* s_full = bar + 4;     // [2]
  uint64_t* s_empty = bar + 6;    // [2]
  uint64_t* acc_full = bar + 8;   // [2]
  uint64_t* acc_empty = bar + 10; // [2], 8 epilogue warps
  uint64_t* w_full = bar + 12;
  uint64_t* w_empty = bar + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 14);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < 14; ++i) mbar_init(smem_u32(&bar[i]), (i == 10 || i == 11) ? 8 : 1);
    *abort_flag = 0;
    abort_flag[2] = 1;  // epilogue "go" flag
    fence_mbar_init();
    tma_prefetch(&tq);
    tma_prefetch(&tg);
    tma_prefetch(&tw);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sS = smem_u32(smem + ReadoutSmem::kS), sW = smem_u32(smem + ReadoutSmem::kW);
  const uint32_t sQG = smem_u32(smem + ReadoutSmem::kQG);
  // units (f, h) head-major, a contiguous range per CTA so W_up changes rarely
  const int units = F * H;
  const int u0 = (int)((long long)blockIdx.x * units / gridDim.x);
  const int u1 = (int)((long long)(blockIdx.x + 1) * units / gridDim.x);
  const int ntile = (T + kRows - 1) / kRows;
  auto head_of = [&](int u) { return u / F; };
  auto frame_of = [&](int u) { return u - (u / F) * F; };

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t ph = 0, w_waits = 0;
      for (int u = u0; u < u1; ++u) {
        const int h = head_of(u), f = frame_of(u);
        if (u == u0 || h != head_of(u - 1)) {
          if (u != u0 && !mbar_wait(smem_u32(w_empty), (w_waits++) & 1, abort_flag, err, kErrWaitProducer)) break;
          mbar_arrive_expect_tx(smem_u32(w_full), kTile);
          for (int b = 0; b < 2; ++b) tma_load_2d(sW + b * kBlk, &tw, smem_u32(w_full), b * 64, h * D);
        }
        bool ok = true;
        for (int t = 0; t < ntile; ++t) {
          if (!mbar_wait(smem_u32(&qg_empty[stage]), ph ^ 1, abort_flag, err, kErrWaitProducer)) {
            ok = false;
            break;
          }
          const uint32_t sq = sQG + stage * 2 * kTile, sg = sq + kTile;
          mbar_arrive_expect_tx(smem_u32(&qg_full[stage]), 2 * kTile);
          for (int b = 0; b < 2; ++b) {
            tma_load_2d(sq + b * kBlk, &tq, smem_u32(&qg_full[stage]), b * 64, ((f * H + h) * T) + t * kRows);
            tma_load_2d(sg + b * kBlk, &tg, smem_u32(&qg_full[stage]), b * 64, f * T + t * kRows);
          }
          if (++stage == 2) {
            stage = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(1, 1, 1, 0, 0, 128, 128);
      int stage = 0, acc = 0, sb = 0;
      uint32_t ph = 0, acc_ph = 0, w_waits = 0;
      bool ok = true;
      for (int u = u0; u < u1 && ok; ++u) {
        const int h = head_of(u);
        const bool last_of_head = (u + 1 == u1) || head_of(u + 1) != h;
        if (u == u0 || h != head_of(u - 1)) {
          if (!mbar_wait(smem_u32(w_full), (w_waits++) & 1, abort_flag, err, kErrWaitMma)) break;
        }
        // state buffer sb serves units u0 + sb, u0 + sb + 2, ...
        if (!mbar_wait(smem_u32(&s_full[sb]), ((u - u0) >> 1) & 1, abort_flag, err, kErrWaitMma)) break;
        const uint32_t ss = sS + sb * kTile;
        for (int t = 0; t < ntile; ++t) {
          if (!mbar_wait(smem_u32(&acc_empty[acc]), acc_ph ^ 1, abort_flag, err, kErrWaitMma) ||
              !mbar_wait(smem_u32(&qg_full[stage]), ph, abort_flag, err, kErrWaitMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sq = sQG + stage * 2 * kTile, sg = sq + kTile;
          const uint32_t d = tmem + acc * 256;
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint32_t off = (k >> 2) * kBlk + (k & 3) * 32;
            mma_f16(d, make_sdesc(sq + off, 16, 1024), make_sdesc(ss + off, 16, 1024), idesc, k > 0 ? 1u : 0u);
            mma_f16(d + 128, make_sdesc(sg + off, 16, 1024), make_sdesc(sW + off, 16, 1024), idesc,
                    k > 0 ? 1u : 0u);
          }
          tc_commit(smem_u32(&qg_empty[stage]));
          tc_commit(smem_u32(&acc_full[acc]));
          if (t == ntile - 1) {
            tc_commit(smem_u32(&s_empty[sb]));
            if (last_of_head) tc_commit(smem_u32(w_empty));
          }
          if (++stage == 2) {
            stage = 0;
            ph ^= 1;
          }
          if (++acc == 2) {
            acc = 0;
            acc_ph ^= 1;
          }
        }
        sb ^= 1;
      }
    }
  } else if (warp < 4) {
    // state builders (64 threads): state[v][k] = bf16(prefix[v][k] dec_b[k] + suffix[v][k] dec_a[k])
    // The 64 builders synchronise on named barrier 1; builder 0 alone waits on the
    // mbarrier and publishes the outcome in shared memory, so a timed-out wait makes all
    // 64 leave together instead of stranding some at the named barrier.
    const int bt = tid - 64;
    volatile int* go = reinterpret_cast<volatile int*>(abort_flag + 1);
    int sb = 0;
    for (int u = u0; u < u1; ++u) {
      const int h = head_of(u), f = frame_of(u);
      if (bt == 0)
        *go = mbar_wait(smem_u32(&s_empty[sb]), (((u - u0) >> 1) & 1) ^ 1, abort_flag, err, kErrWaitOther) ? 1 : 0;
      asm volatile("bar.sync 1, 64;" ::: "memory");
      if (!*go) break;
      // alpha-bridge decays (branch.py:385-390) of this thread's fixed chunk of 8 k
      // (every element it writes has k = (bt & 15) * 8 + q)
      // f is the frame within this call's frames; the gather works in clip frames fg
      const int fg = f0 + f;
      const int raw_lo = lo_arr[fg], raw_hi = hi_arr[fg];
      const int lo = max(raw_lo, 0), hi = min(raw_hi, F_all - 1);
      const bool has_before = raw_lo - 1 >= 0, has_after = raw_hi + 1 < F_all;
      const int kc = (bt & 15) * 8;
      float dec_b[8], dec_a[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float lb = 0.f, la = 0.f;
        if (use_alpha) {
          for (int j = lo; j <= fg; ++j) lb += __logf(fmaxf(alpha[((long long)j * H + h) * D + kc + q], 1e-12f));
          for (int j = fg; j <= hi; ++j) la += __logf(fmaxf(alpha[((long long)j * H + h) * D + kc + q], 1e-12f));
        }
        dec_b[q] = __expf(lb);
        dec_a[q] = __expf(la);
      }
      const float* pb = has_before ? prefix + ((long long)(lo - 1) * H + h) * D * D
                                   : (s0 ? s0 + (long long)h * D * D : nullptr);
      const float* pa = has_after ? suffix + ((long long)(hi + 1) * H + h) * D * D
                                  : (s0 ? s0 + (long long)h * D * D : nullptr);
      const uint32_t ss = sS + sb * kTile;
#pragma unroll 4
      for (int i = 0; i < 32; ++i) {
        const int e = bt + 64 * i;
        const int v = e >> 4, c = e & 15;  // 16 chunks of 8 k per row
        float val[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) val[q] = 0.f;
        if (pb) {
          const float4 a0 = *reinterpret_cast<const float4*>(pb + v * D + c * 8);
          const float4 a1 = *reinterpret_cast<const float4*>(pb + v * D + c * 8 + 4);
          const float tv[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
          for (int q = 0; q < 8; ++q) val[q] += tv[q] * dec_b[q];
        }
        if (pa) {
          const float4 a0 = *reinterpret_cast<const float4*>(pa + v * D + c * 8);
          const float4 a1 = *reinterpret_cast<const float4*>(pa + v * D + c * 8 + 4);
          const float tv[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
          for (int q = 0; q < 8; ++q) val[q] += tv[q] * dec_a[q];
        }
        const uint32_t addr = ss + (c >> 3) * kBlk + v * 128 + (((c & 7) ^ (v & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(pack_bf16(val[0], val[1])),
                     "r"(pack_bf16(val[2], val[3])), "r"(pack_bf16(val[4], val[5])), "r"(pack_bf16(val[6], val[7]))
                     : "memory");
      }
      fence_proxy_async_smem();
      asm volatile("bar.sync 1, 64;" ::: "memory");
      if (bt == 0) mbar_arrive(smem_u32(&s_full[sb]));
      sb ^= 1;
    }
  } else {
    // epilogue: 8 warps; warp w reads TMEM lane quadrant w % 4 (32 token rows) and column
    // half ch = (w - 4) / 4 (64 of the 128 values).  The RMSNorm sum of squares of a row is
    // combined across the two halves through shared memory (named barrier 2, 256 threads).
    const int quad = warp & 3, ch = (warp - 4) >> 2;
    const int row = quad * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    float* ssp = reinterpret_cast<float*>(smem + ReadoutSmem::kSsq);  // [2 acc][2 halves][128 rows]
    volatile int* epi_go = reinterpret_cast<volatile int*>(abort_flag + 2);
    const float* nw = norm_w + ch * 64;
    int acc = 0;
    uint32_t acc_ph = 0;
    bool ok = true;
    for (int u = u0; u < u1 && ok; ++u) {
      const int h = head_of(u), f = frame_of(u);
      const float* bias = og_bias + h * D + ch * 64;
      for (int t = 0; t < ntile; ++t) {
        // warp-uniform wait; a failed wait still joins the named barrier, then all leave
        const bool okw = __all_sync(0xffffffffu,
                                    mbar_wait(smem_u32(&acc_full[acc]), acc_ph, abort_flag, err, kErrWaitEpilogue));
        uint32_t r[64];
        float ssq = 0.f;
        const uint32_t tb = tmem + lane_base + acc * 256 + ch * 64;
        if (okw) {
          tc_fence_after();
          tmem_ld32(tb, *reinterpret_cast<uint32_t(*)[32]>(r));
          tmem_ld32(tb + 32, *reinterpret_cast<uint32_t(*)[32]>(r + 32));
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            const float x = bf16_round(__uint_as_float(r[i]));
            r[i] = __float_as_uint(x);
            ssq = fmaf(x, x, ssq);
          }
          ssp[(acc * 2 + ch) * 128 + row] = ssq;
        } else {
          *epi_go = 0;
        }
        asm volatile("bar.sync 2, 256;" ::: "memory");
        if (!*epi_go) {
          ok = false;
          break;
        }
        const float* sp = ssp + acc * 2 * 128 + row;
        const float inv = rsqrtf((sp[0] + sp[128]) / (float)D + 1e-6f);
        const int tok = t * kRows + row;
        __nv_bfloat16* dst = out + (out_row0 + (long long)f * T + tok) * ld_out + h * D + ch * 64;
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          uint32_t gr[32];
          tmem_ld32(tb + 128 + c2 * 32, gr);
          tmem_ld_wait();
          if (c2 == 1) {  // every TMEM read of this accumulator is done
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&acc_empty[acc]));
          }
          if (tok < T) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              // norm weights and gate biases of these 8 columns as two 16-byte loads each
              const int v0 = c2 * 32 + i;
              const float4 w0 = *reinterpret_cast<const float4*>(nw + v0);
              const float4 w1 = *reinterpret_cast<const float4*>(nw + v0 + 4);
              const float4 b0 = *reinterpret_cast<const float4*>(bias + v0);
              const float4 b1 = *reinterpret_cast<const float4*>(bias + v0 + 4);
              const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
              const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
              float o[8];
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                const float nv = bf16_round(__uint_as_float(r[v0 + q]) * inv * wv[q]);
                // nv * sigmoid(g + b) = nv / (1 + 2^(-(g + b) log2 e))
                const float e = ex2_ftz(-(__uint_as_float(gr[i + q]) + bv[q]) * 1.4426950408889634f);
                o[q] = nv * rcp_ftz(1.0f + e);
              }
              uint4 pk;
              pk.x = pack_bf16(o[0], o[1]);
              pk.y = pack_bf16(o[2], o[3]);
              pk.z = pack_bf16(o[4], o[5]);
              pk.w = pack_bf16(o[6], o[7]);
              *reinterpret_cast<uint4*>(dst + c2 * 32 + i) = pk;
            }
          }
        }
        if (++acc == 2) {
          acc = 0;
          acc_ph ^= 1;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) abort_drain();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------------- scan
// Bidirectional scan on the tensor cores: one CTA per (head, direction) keeps the 128 x 128
// state in TMEM and runs, per frame,
//     u = B_t + s o alpha_t          (warps 0-3, thread = state row, from TMEM + HBM)
//     s = u (I + A_t)^-1             (warp 4: 24 tcgen05 MMAs)
// The product is done in three bf16 passes, u_hi inv_hi + u_hi inv_lo + u_lo inv_hi with
// x = hi + lo (hi = bf16(x), lo = bf16(x - hi)), accumulated in fp32: 16 significant bits per
// operand, so the state carries ~1e-5 relative error per frame (it is rounded to bf16 for the
// readout).  The inverse halves come from vdn_delta_factor; the next frame's are loaded by
// TMA while the current frame is multiplied.
// kSana (delta_rule "sana_scaled", branch.py:163-177): the matrix is M = I - A/L (halves from
// vdn_sana_factor) and the injection is added after the product,
//     u = s o alpha_t,   s = u M_t + inj_scale B_t,
// so the B row a thread needs at step t is that of the frame whose product it reads back.
// smem: 2 stages x (inv hi, inv lo) + (u hi, u lo) = 6 x 32 KB dynamic, plus 22 KB static per
// CTA: each state warp's alpha row (double-buffered) and its 32 x 32 transpose tile, through
// which the B rows arrive and the state rows leave as whole 128-byte row pieces.
struct ScanSmem {
  static constexpr int kInv = 0, kU = 4 * kTile, kBar = 6 * kTile;
  static constexpr int kBytes = kBar + 256 + 1024;
};
constexpr int kScanThreads = 160;
constexpr int kXPitch = 36;  // floats per row of the scan's transpose tiles

template <bool kSana>
__global__ void __launch_bounds__(kScanThreads, 1)
    scan_tc_kernel(const __grid_constant__ CUtensorMap tinv, const float* __restrict__ Bm,
                   const float* __restrict__ alpha, const float* __restrict__ s0, int F, int F_inv, int H,
                   float inj_scale, float* __restrict__ prefix, float* __restrict__ suffix, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // per row warp, double-buffered by step: the current frame's alpha row
  __shared__ __align__(16) float alpha_s[4][2][D];
  // per row warp: a 32 x 32 fp32 tile (rows padded to kXPitch floats, so the 16-byte accesses
  // of a quarter warp hit distinct banks whether it walks a row or a column of rows) that
  // turns coalesced B pieces into thread rows and thread rows into coalesced state pieces
  __shared__ __align__(16) float xpose[4][32][kXPitch];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + ScanSmem::kBar);
  uint64_t* inv_full = bar;       // [2]
  uint64_t* inv_empty = bar + 2;  // [2]
  uint64_t* a_full = bar + 4;     // 4 row warps
  uint64_t* mma_done = bar + 5;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.x, dir = blockIdx.y;
  if (tid == 0) {
    for (int i = 0; i < 6; ++i) mbar_init(smem_u32(&bar[i]), i == 4 ? 4 : 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch(&tinv);
  }
  if (warp == 4) {
    tmem_alloc(smem_u32(tmem_slot), 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sInv = smem_u32(smem + ScanSmem::kInv), sU = smem_u32(smem + ScanSmem::kU);
  auto frame = [&](int step) { return dir == 0 ? step : F - 1 - step; };
  float* dst_all = dir == 0 ? prefix : suffix;

  if (warp == 4) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(1, 1, 1, 0, 0, 128, 128);
      const int lo_rows = F_inv * H * D;  // the lo halves follow the hi halves
      auto issue = [&](int step) {
        const int st = step & 1;
        if (!mbar_wait(smem_u32(&inv_empty[st]), ((step >> 1) & 1) ^ 1, abort_flag, err, kErrWaitProducer))
          return false;
        const int row = (frame(step) * H + h) * D;
        const uint32_t hi = sInv + st * 2 * kTile, lo = hi + kTile;
        mbar_arrive_expect_tx(smem_u32(&inv_full[st]), 2 * kTile);
        for (int b = 0; b < 2; ++b) {
          tma_load_2d(hi + b * kBlk, &tinv, smem_u32(&inv_full[st]), b * 64, row);
          tma_load_2d(lo + b * kBlk, &tinv, smem_u32(&inv_full[st]), b * 64, lo_rows + row);
        }
        return true;
      };
      bool ok = issue(0);
      for (int step = 0; step < F && ok; ++step) {
        const int st = step & 1;
        if (step + 1 < F && !issue(step + 1)) break;
        if (!mbar_wait(smem_u32(&inv_full[st]), (step >> 1) & 1, abort_flag, err, kErrWaitMma) ||
            !mbar_wait(smem_u32(a_full), step & 1, abort_flag, err, kErrWaitMma))
          break;
        tc_fence_after();
        const uint32_t ihi = sInv + st * 2 * kTile, ilo = ihi + kTile, uhi = sU, ulo = sU + kTile;
        const uint32_t ops[3][2] = {{uhi, ihi}, {uhi, ilo}, {ulo, ihi}};
#pragma unroll
        for (int pass = 0; pass < 3; ++pass)
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint32_t off = (k >> 2) * kBlk + (k & 3) * 32;
            mma_f16(tmem, make_sdesc(ops[pass][0] + off, 16, 1024), make_sdesc(ops[pass][1] + off, 16, 1024), idesc,
                    (pass > 0 || k > 0) ? 1u : 0u);
          }
        tc_commit(smem_u32(&inv_empty[st]));
        tc_commit(smem_u32(mma_done));
      }
    }
  } else {
    // state rows: thread i = row i = TMEM lane i
    const int i = tid;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    bool ok = true;
    for (int step = 0; step < F && ok; ++step) {
      const int t = frame(step);
      // this frame's B row (kSana: the previous frame's) does not depend on the previous state:
      // it is in registers before the wait for the previous step's MMA, off the dependent
      // chain of the recurrence
      // Loaded coalesced: for chunk c (columns 32c ..) lane l holds columns 32c + 4 (l % 8) .. +3
      // of the warp's rows 4k + l / 8 (k < 8), so each load instruction reads four whole
      // 128-byte row pieces; the warp's xpose tile turns them into this thread's own row.
      const float* bmat = Bm + ((long long)(kSana ? frame(step > 0 ? step - 1 : 0) : t) * H + h) * D * D;
      const int prow = warp * 32 + (lane >> 3), pcol = (lane & 7) * 4;
      float4 bv[D / 32][8];
#pragma unroll
      for (int c = 0; c < D / 32; ++c)
#pragma unroll
        for (int k = 0; k < 8; ++k)
          bv[c][k] = (kSana && step == 0) ? make_float4(0.f, 0.f, 0.f, 0.f)
                                          : __ldg(reinterpret_cast<const float4*>(bmat + (long long)(prow + 4 * k) * D +
                                                                                  c * 32 + pcol));
      if (step + 1 < F) {  // the next frame's B row into L2 meanwhile
        const float* nb = Bm + (((long long)frame(step + 1) * H + h) * D + i) * D;
#pragma unroll
        for (int q = 0; q < 4; ++q) asm volatile("prefetch.global.L2 [%0];" ::"l"(nb + q * 32));
      }
      // the frame's alpha row, a 16-byte piece per lane, is loaded before the wait too and
      // shared through this warp's own row of alpha_s after it (warp-synchronous only)
      const float4 a_piece = __ldg(reinterpret_cast<const float4*>(alpha + ((long long)t * H + h) * D) + lane);
      if (step > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(mma_done), (step - 1) & 1, abort_flag, err, kErrWaitOther));
        if (!ok) break;
        tc_fence_after();
      }
      float* al = alpha_s[warp][step & 1];
      reinterpret_cast<float4*>(al)[lane] = a_piece;
      __syncwarp();
      // the previous frame's state goes out by the same tile, as whole 128-byte row pieces
      float* prev = step > 0 ? dst_all + ((long long)frame(step - 1) * H + h) * D * D : nullptr;
      float* xt = &xpose[warp][0][0];
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        // this chunk of B: the lanes' pieces into the tile, then this thread's row out of it
#pragma unroll
        for (int k = 0; k < 8; ++k) *reinterpret_cast<float4*>(xt + (4 * k + (lane >> 3)) * kXPitch + pcol) = bv[c][k];
        __syncwarp();
        float4 bq[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) bq[q] = *reinterpret_cast<const float4*>(xt + lane * kXPitch + 4 * q);
        __syncwarp();
        float sv[32];
        if (step == 0) {
#pragma unroll
          for (int q = 0; q < 32; ++q) sv[q] = s0 ? s0[((long long)h * D + i) * D + c * 32 + q] : 0.f;
        } else {
          uint32_t r[32];
          tmem_ld32(tmem + lane_base + c * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < 32; ++q) sv[q] = __uint_as_float(r[q]);
          if (kSana) {
#pragma unroll
            for (int q = 0; q < 32; q += 4) {
              const float4 b4 = bq[q / 4];
              sv[q] = fmaf(inj_scale, b4.x, sv[q]);
              sv[q + 1] = fmaf(inj_scale, b4.y, sv[q + 1]);
              sv[q + 2] = fmaf(inj_scale, b4.z, sv[q + 2]);
              sv[q + 3] = fmaf(inj_scale, b4.w, sv[q + 3]);
            }
          }
          // this thread's row into the tile, then whole row pieces out to the previous frame
#pragma unroll
          for (int q = 0; q < 32; q += 4)
            *reinterpret_cast<float4*>(xt + lane * kXPitch + q) = make_float4(sv[q], sv[q + 1], sv[q + 2], sv[q + 3]);
          __syncwarp();
#pragma unroll
          for (int k = 0; k < 8; ++k)
            *reinterpret_cast<float4*>(prev + (long long)(prow + 4 * k) * D + c * 32 + pcol) =
                *reinterpret_cast<const float4*>(xt + (4 * k + (lane >> 3)) * kXPitch + pcol);
          __syncwarp();
        }
        // u = B + s o alpha, split into bf16 hi + lo, written K-major swizzled (8 values per 16 B)
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          const int k0 = c * 32 + q8 * 8;
          const float4 b0 = bq[q8 * 2];
          const float4 b1 = bq[q8 * 2 + 1];
          const float4 a0 = *reinterpret_cast<const float4*>(al + k0);
          const float4 a1 = *reinterpret_cast<const float4*>(al + k0 + 4);
          const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
          const float aa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
          uint32_t hp[4], lp[4];
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            const float u0 = kSana ? sv[q8 * 8 + e] * aa[e] : fmaf(sv[q8 * 8 + e], aa[e], bb[e]);
            const float u1 = kSana ? sv[q8 * 8 + e + 1] * aa[e + 1] : fmaf(sv[q8 * 8 + e + 1], aa[e + 1], bb[e + 1]);
            const __nv_bfloat162 h2 = __floats2bfloat162_rn(u0, u1);
            const float2 hf = __bfloat1622float2(h2);
            hp[e / 2] = *reinterpret_cast<const uint32_t*>(&h2);
            lp[e / 2] = pack_bf16(u0 - hf.x, u1 - hf.y);
          }
          const int ch = k0 >> 3;  // 16-byte chunk of the row, 0..15
          const uint32_t off = (ch >> 3) * kBlk + i * 128 + (((ch & 7) ^ (i & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sU + off), "r"(hp[0]), "r"(hp[1]), "r"(hp[2]),
                       "r"(hp[3])
                       : "memory");
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sU + kTile + off), "r"(lp[0]), "r"(lp[1]),
                       "r"(lp[2]), "r"(lp[3])
                       : "memory");
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(a_full));
    }
    if (ok && __all_sync(0xffffffffu, mbar_wait(smem_u32(mma_done), (F - 1) & 1, abort_flag, err, kErrWaitOther))) {
      tc_fence_after();
      float* last = dst_all + (((long long)frame(F - 1) * H + h) * D + i) * D;
      const float* blast = Bm + (((long long)frame(F - 1) * H + h) * D + i) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + c * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int q = 0; q < 32; q += 4) {
          float4 v = make_float4(__uint_as_float(r[q]), __uint_as_float(r[q + 1]), __uint_as_float(r[q + 2]),
                                 __uint_as_float(r[q + 3]));
          if (kSana) {
            const float4 b4 = __ldg(reinterpret_cast<const float4*>(blast + c * 32 + q));
            v = make_float4(fmaf(inj_scale, b4.x, v.x), fmaf(inj_scale, b4.y, v.y), fmaf(inj_scale, b4.z, v.z),
                            fmaf(inj_scale, b4.w, v.w));
          }
          *reinterpret_cast<float4*>(last + c * 32 + q) = v;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) abort_drain();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

}  // namespace branch_tc
}  // namespace vdn

extern "C" {

// Frame statistics on tensor cores (head_dim 128).  K, V: FHSD [F, H, T, 128] bf16;
// beta logits [F*T, ld_beta] fp32 (column beta_col0 + h); A, B out [F, H, 128, 128] fp32.
// Replaces branch.py:197-282 (frame_statistics).
int vdn_frame_stats_tc(const void* K, const void* V, int F, int H, int T, const float* beta_logits, long long ld_beta,
                       int beta_col0, float* A, float* B, int* dev_err, void* stream) {
  using namespace vdn::branch_tc;
  if (!K || !V || !beta_logits || !A || !B || F <= 0 || H <= 0 || T <= 0) return vdn::kBadArgument;
  if (!vdn::aligned16(A) || !vdn::aligned16(B)) return vdn::kMisaligned;  // float4 row stores
  CUtensorMap tk, tv;
  const uint64_t rows = (uint64_t)F * H * T;
  int rc = vdn::make_tmap_2d(&tk, K, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, rows, D, 64, 128);
  if (rc) return rc;
  rc = vdn::make_tmap_2d(&tv, V, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, rows, D, 64, 128);
  if (rc) return rc;
  if (!vdn::smem_optin((const void*)frame_stats_tc_kernel, StatsSmem::kBytes)) return vdn::kLaunchFailed;
  const int units = F * H;
  const int grid = units < vdn::sm_count() ? units : vdn::sm_count();
  frame_stats_tc_kernel<<<grid, kStatsThreads, StatsSmem::kBytes, reinterpret_cast<cudaStream_t>(stream)>>>(
      tk, tv, F, H, T, beta_logits, ld_beta, beta_col0, A, B, dev_err);
  vdn::count_launch();
  return vdn::launch_status();
}

// Readout on tensor cores (head_dim 128) of the F frames f0 .. f0+F-1 of a clip of F_all
// frames: Q FHSD [F, H, T, 128] bf16 and og_down [F*T, 128] bf16 (bf16-rounded x W_og_down^T)
// hold those frames' rows; og_up [H*128, 128] bf16 with bias og_bias [H*128] fp32;
// prefix/suffix [F_all, H, 128, 128] fp32; alpha [F_all, H, 128]; s0 [H, 128, 128] or NULL;
// lo/hi [F_all] raw window bounds.  Writes out[out_row0 + f*T + s, h*128 + v] (bf16).
// Replaces branch.py:345-396 (gather), :780 (readout), :494-530 (epilogue), :754-758 (gate).
int vdn_readout_tc(const void* Q, int F, int H, int T, const float* prefix, const float* suffix, const float* alpha,
                   const float* s0, const int* lo, const int* hi, int use_alpha, const float* norm_w,
                   const void* og_down, const void* og_up, const float* og_bias, void* out, long long ld_out,
                   long long out_row0, int f0, int F_all, int* dev_err, void* stream) {
  using namespace vdn::branch_tc;
  if (!Q || !prefix || !suffix || !alpha || !lo || !hi || !norm_w || !og_down || !og_up || !og_bias || !out)
    return vdn::kBadArgument;
  if (F <= 0 || f0 < 0 || F_all < f0 + F) return vdn::kBadArgument;
  if ((ld_out * 2) % 16 || !vdn::aligned16(out) || !vdn::aligned16(prefix) || !vdn::aligned16(suffix) ||
      (s0 && !vdn::aligned16(s0)) || !vdn::aligned16(norm_w) || !vdn::aligned16(og_bias))
    return vdn::kMisaligned;  // 16-byte output vectors, float4 state, norm-weight and bias loads
  CUtensorMap tq, tg, tw;
  int rc = vdn::make_tmap_2d(&tq, Q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, (uint64_t)F * H * T, D, 64, 128);
  if (rc) return rc;
  rc = vdn::make_tmap_2d(&tg, og_down, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, (uint64_t)F * T, D, 64, 128);
  if (rc) return rc;
  rc = vdn::make_tmap_2d(&tw, og_up, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, (uint64_t)H * D, D, 64, 128);
  if (rc) return rc;
  if (!vdn::smem_optin((const void*)readout_tc_kernel, ReadoutSmem::kBytes)) return vdn::kLaunchFailed;
  const int units = F * H;
  const int grid = units < vdn::sm_count() ? units : vdn::sm_count();
  readout_tc_kernel<<<grid, kReadoutThreads, ReadoutSmem::kBytes, reinterpret_cast<cudaStream_t>(stream)>>>(
      tq, tg, tw, F, H, T, prefix, suffix, alpha, s0, lo, hi, use_alpha, norm_w, og_bias,
      reinterpret_cast<__nv_bfloat16*>(out), ld_out, out_row0, f0, F_all, dev_err);
  vdn::count_launch();
  return vdn::launch_status();
}

// Bidirectional scan on tensor cores (head_dim 128): inv_split = the bf16 hi halves of the
// F_inv inverses [F_inv, H, 128, 128] followed by the lo halves (vdn_delta_factor's
// inv_split output, or vdn_sana_factor's M_split with inj_scale > 0); B [F_inv, H, 128, 128]
// fp32 (frames 0..F-1 used); alpha [F, H, 128]; s0 [H, 128, 128] or NULL; prefix/suffix
// [F, H, 128, 128] fp32.  Replaces branch.py:297-312 (run_scans_*), with T and Inj folded as
// in vdn_bidir_scan.
int vdn_bidir_scan_tc(const void* inv_split, const float* B, const float* alpha, const float* s0, int F, int F_inv,
                      int H, float inj_scale, float* prefix, float* suffix, int* dev_err, void* stream) {
  using namespace vdn::branch_tc;
  if (!inv_split || !B || !alpha || !prefix || !suffix || F <= 0 || F > F_inv || H <= 0 || inj_scale < 0.f)
    return vdn::kBadArgument;
  if (!vdn::aligned16(B) || !vdn::aligned16(alpha) || !vdn::aligned16(prefix) || !vdn::aligned16(suffix))
    return vdn::kMisaligned;  // float4 rows
  CUtensorMap tinv;
  int rc = vdn::make_tmap_2d(&tinv, inv_split, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, (uint64_t)2 * F_inv * H * D, D,
                             64, 128);
  if (rc) return rc;
  if (!vdn::smem_optin((const void*)scan_tc_kernel<false>, ScanSmem::kBytes) ||
      !vdn::smem_optin((const void*)scan_tc_kernel<true>, ScanSmem::kBytes))
    return vdn::kLaunchFailed;
  auto kernel = inj_scale > 0.f ? scan_tc_kernel<true> : scan_tc_kernel<false>;
  kernel<<<dim3(H, 2), kScanThreads, ScanSmem::kBytes, reinterpret_cast<cudaStream_t>(stream)>>>(
      tinv, B, alpha, s0, F, F_inv, H, inj_scale, prefix, suffix, dev_err);
  vdn::count_launch();
  return vdn::launch_status();
}

}  // extern "C"
