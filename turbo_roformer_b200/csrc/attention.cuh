// Exact-softmax gated attention on tcgen05 (flash-style, online softmax with exact rescaling).
//
// Replaces the reference's AVX-512 `attention` kernel (LoggeL/turbo-roformer
// src/turbo_roformer/csrc/kernels.cpp:255-388): per (sequence, head) S = Q K^T (scale folded into W_q),
// softmax over the keys, O = P V, then x sigmoid gate, head merge and scatter back to token order.
// The reference keeps whole score rows (two passes); here a CTA owns two 128-row query tiles (A, B)
// and streams 128-key tiles:
//   * S = Q K^T (both operands in shared memory) lands in TMEM. The softmax warps of the tile read the
//     whole score row into registers at once, which frees the S columns: the next key tile's S is
//     issued right then and runs on the tensor core while this tile's exponentials are computed.
//   * Unnormalised 16-bit P goes to its own TMEM columns and the tensor core computes O += P V with P
//     read straight from TMEM (no shared-memory round trip for P). O accumulates in TMEM.
//   * The running row maximum is only raised when a tile's maximum exceeds it by more than 2^8 (then O
//     and the row sum are rescaled in place); P <= 2^8 keeps 16-bit P exact enough and the final O / l
//     is the exact softmax average.
//   * Each query tile has its own MMA-issuing thread (warps 1 and 2), so the two tiles' products are
//     issued independently: next S once the softmax has taken the previous one, P V once P is written.
//   * At head dim 64 the exponentials, not the products, set the pace (16 ex2 per clock per SM on the
//     MUFU pipe against 8192 tensor flops): one key pair in four is exponentiated by a polynomial on the
//     FMA pipe instead (ex2_poly2), and the softmax warps take the registers the TMA / MMA warps do not
//     need (setmaxnreg), so the whole score row and its packed P fit without spills.
//   * Persistent CTAs walk the work items; Q is double buffered so the next item's first products
//     start while the current item's epilogue runs.
//
// Layout: Q, K, V are [BH, L, 64] 16-bit, row-major, unpadded; the 3-D TMA maps zero-fill rows >= L.
//   time mode (mode 0): sequences = (batch, band, head), L = T frames; an item = one sequence and two
//                       consecutive 128-row query tiles; every key tile serves both query tiles.
//   freq mode (mode 1): sequences = (batch, frame, head), L = bands <= 64; a query tile holds two
//                       sequences (block-diagonal mask), an item = four sequences, each tile has its own
//                       single key tile.
// Roles (384 threads, three warpgroups): warp 0 TMA, warp 1 MMA issuer of tile A + TMEM owner, warp 2 MMA
// issuer of tile B, warp 3 idle (warps 0-3 release registers); warps 4-7 softmax + epilogue of tile A,
// warps 8-11 of tile B (thread = query row; warp w reads TMEM lanes 32 (w % 4) ..).
#pragma once

#include "gemm.cuh"  // store32
#include "sm100.cuh"

namespace trc {

constexpr int kAttnThreads = 384;
// Time mode: registers per thread after setmaxnreg for warps 0-3 and for the softmax warpgroups. The
// launch gives every thread the same count R (168 at 384 threads); the split needs
// 4 * 32 * kAttnRegsLow + 8 * 32 * kAttnRegsHigh <= 384 * R, or the increase would wait forever
// (launch_attention checks R before every time-mode launch).
constexpr int kAttnRegsLow = 56;
constexpr int kAttnRegsHigh = 216;
// Key/value stages. Frequency mode loads one stage per tile and item (tile A, tile B, tile A, ...): with an
// even stage count, stage (2 item + tile) % kAttnKvStages is only ever used by that one tile, so each
// tile's MMA issuer waits on every phase of its stages in order. With an odd count the tiles would share
// stages, and a tile running an item ahead could wait on a stage whose previous phase (the other tile's
// load) had not completed yet, where a parity wait cannot tell the two phases apart.
constexpr int kAttnKvStages = 4;
static_assert(kAttnKvStages % 2 == 0, "frequency mode needs per-tile stages");

struct AttnArgs {
  int num_items;  // work items
  int q_pairs;    // time: query-tile pairs per sequence
  int n_kv;       // time: key tiles per sequence
  int L;          // valid length of every sequence
  int BH;         // number of sequences
  int mode;       // 0 time, 1 freq
  int T, F;       // frames, bands (per batch item)
  const float* G;  // gates [tokens][8]
  void* O;         // [tokens][512] 16-bit
  int* err;
};

struct AttnSmem {
  static constexpr int kTile = 128 * 64 * 2;  // 16 KB: 128 rows x 64 dims
  static constexpr int kQ = 0;                 // [2 buffers][2 tiles]
  static constexpr int kKV = kQ + 4 * kTile;   // [stages][K, V]
  static constexpr int kScale = kKV + 2 * kAttnKvStages * kTile;  // [2 tiles][128 rows] gate / l (fp32)
  static constexpr int kBar = kScale + 2 * 128 * 4;
  static constexpr int kBytes = kBar + 512 + 1024;
  static_assert(kBytes <= 232448, "shared memory per CTA");
};

// TMEM columns (all 512): S_A [0,128), S_B [128,256), P_A [256,320), P_B [320,384) (16-bit pairs),
// O_A [384,448), O_B [448,512)
__device__ __forceinline__ uint32_t tmem_col_s(int x) { return (uint32_t)x * 128u; }
__device__ __forceinline__ uint32_t tmem_col_p(int x) { return 256u + (uint32_t)x * 64u; }
__device__ __forceinline__ uint32_t tmem_col_o(int x) { return 384u + (uint32_t)x * 64u; }
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P stays <= 2^8

// 2^x for a pair of fp32 values on the FMA pipe (no MUFU): x = j + f with j = round(x) (the 1.5 * 2^23
// rounding constant), 2^f on [-1/2, 1/2] by a degree-3 polynomial fitted here for minimum relative error
// (Chebyshev-node least squares with Lawson reweighting; max relative error 7.5e-5, below half an fp16
// ulp), and j added to the exponent field. x is clamped at -126 so the exponent field never wraps; the
// inputs here are <= 2^8 and results below 2^-24 flush to zero in the 16-bit P anyway.
__device__ __forceinline__ float2 ex2_poly2(float2 x) {
  x = make_float2(fmaxf(x.x, -126.f), fmaxf(x.y, -126.f));
  const float2 round_c = make_float2(12582912.0f, 12582912.0f);
  const float2 t = __fadd2_rn(x, round_c);
  const float2 j = __fadd2_rn(t, make_float2(-12582912.0f, -12582912.0f));
  const float2 f = __fadd2_rn(x, make_float2(-j.x, -j.y));
  float2 p = __ffma2_rn(make_float2(0.0551716648f, 0.0551716648f), f, make_float2(0.2426111251f, 0.2426111251f));
  p = __ffma2_rn(p, f, make_float2(0.6932609677f, 0.6932609677f));
  p = __ffma2_rn(p, f, make_float2(0.9999280572f, 0.9999280572f));
  // the low mantissa bits of t hold j: shifted into the exponent field they multiply p by 2^j
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

// kFreq: frequency mode (compiled separately, so each mode gets its own register allocation); it must
// equal args.mode == 1.
template <typename TIn, bool kFreq>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                     const __grid_constant__ CUtensorMap map_v, const __grid_constant__ AttnArgs args) {
  using S = AttnSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBar);
  uint64_t* q_full = bars;                   // [2] per Q buffer
  uint64_t* q_empty = q_full + 2;            // [2]
  uint64_t* kv_full = q_empty + 2;           // [stages]
  uint64_t* kv_empty = kv_full + kAttnKvStages;
  uint64_t* s_full = kv_empty + kAttnKvStages;  // [2] per query tile: S in TMEM (MMA commit)
  uint64_t* s_free = s_full + 2;                // [2] S read into registers (one arrive per softmax warp)
  uint64_t* p_full = s_free + 2;                // [2] P written, O rescaled (one arrive per softmax warp)
  uint64_t* p_free = p_full + 2;                // [2] O += P V done: P reusable, O current (MMA commit)
  uint64_t* o_free = p_free + 2;                // [2] epilogue has read O (one arrive per softmax warp)
  uint64_t* drain = o_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr bool freq = kFreq;
  const int nsteps = freq ? 1 : args.n_kv;       // key tiles per query tile and item
  const int kv_per_item = freq ? 2 : args.n_kv;  // key/value loads per item

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&q_full[b], 1);
      mbar_init(&q_empty[b], 2);
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], 4);
      mbar_init(&p_full[b], 4);
      mbar_init(&p_free[b], 1);
      mbar_init(&o_free[b], 4);
    }
    for (int s = 0; s < kAttnKvStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], freq ? 1 : 2);  // time mode: both query tiles read every stage
    }
    mbar_init(drain, 2);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_k);
    tma_prefetch_desc(&map_v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp < 4) {
  if constexpr (!kFreq) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kAttnRegsLow) : "memory");
  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int kvc = 0, local = 0, q_issued = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < args.num_items && ok; item += gridDim.x, ++local) {
        int bh, q0;
        if (freq) {
          bh = 4 * item;
          q0 = 0;
        } else {
          bh = item / args.q_pairs;
          q0 = (item - bh * args.q_pairs) * 256;
        }
        const int qb = local & 1;
        if (!mbar_wait(&q_empty[qb], ((uint32_t)(local >> 1) & 1) ^ 1, args.err, kErrWaitProducer, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&q_full[qb], 2 * S::kTile);
        uint8_t* qbuf = smem + S::kQ + qb * 2 * S::kTile;
        if (freq) {
          tma_load_3d(qbuf, &map_q, &q_full[qb], 0, 0, bh);
          tma_load_3d(qbuf + S::kTile, &map_q, &q_full[qb], 0, 0, bh + 2);
        } else {
          tma_load_3d(qbuf, &map_q, &q_full[qb], 0, q0, bh);
          tma_load_3d(qbuf + S::kTile, &map_q, &q_full[qb], 0, q0 + 128, bh);
        }
        ++q_issued;
        for (int j = 0; j < kv_per_item; ++j) {
          const int st = kvc % kAttnKvStages;
          const uint32_t u = (uint32_t)(kvc / kAttnKvStages);
          if (!mbar_wait(&kv_empty[st], (u & 1) ^ 1, args.err, kErrWaitProducer, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* kb = smem + S::kKV + st * 2 * S::kTile;
          mbar_arrive_expect_tx(&kv_full[st], 2 * S::kTile);
          const int row = freq ? 0 : j * 128;
          const int seq = freq ? bh + 2 * j : bh;
          tma_load_3d(kb, &map_k, &kv_full[st], 0, row, seq);
          tma_load_3d(kb + S::kTile, &map_v, &kv_full[st], 0, row, seq);
          ++kvc;
        }
      }
      // let the last issued copies land before the CTA may exit (they are consumed already unless an
      // error aborted the pipeline); bounded like every wait
      const uint64_t t0 = global_ns();
      for (int k = max(0, kvc - kAttnKvStages); k < kvc; ++k)
        while (!mbar_try_wait(&kv_full[k % kAttnKvStages], (uint32_t)(k / kAttnKvStages) & 1) &&
               global_ns() - t0 < kWaitLimitNs) {
        }
      for (int k = max(0, q_issued - 2); k < q_issued; ++k)
        while (!mbar_try_wait(&q_full[k & 1], (uint32_t)(k >> 1) & 1) && global_ns() - t0 < kWaitLimitNs) {
        }
    }
  } else if (warp == 1 || warp == 2) {
    // ------------------------------------------------------------------ MMA issuers, one per query tile
    if (lane == 0) {
      const int x = warp == 1 ? 0 : 1;
      const uint32_t idesc_qk = idesc_f16(128, 128, OperandType<TIn>::kFormat, 0, 0);
      const uint32_t idesc_pv = idesc_f16(128, 64, OperandType<TIn>::kFormat, 0, 1);  // V is MN-major
      const uint32_t tS = tmem_base + tmem_col_s(x), tP = tmem_base + tmem_col_p(x),
                     tO = tmem_base + tmem_col_o(x);
      // shared-memory descriptors of stage 0 / Q buffer 0; other stages, buffers and K steps only move the
      // 16-byte-unit start address in the low bits (every address is below 256 KB, so no carry)
      const uint64_t q_desc0 = sdesc_sw128(smem_u32(smem + S::kQ + x * S::kTile), 16, 1024);
      const uint64_t k_desc0 = sdesc_sw128(smem_u32(smem + S::kKV), 16, 1024);
      const uint64_t v_desc0 = sdesc_sw128(smem_u32(smem + S::kKV + S::kTile), 8192, 1024);
      constexpr uint32_t kStep = (2 * S::kTile) >> 4;  // one KV stage or one Q buffer
      int kvc = 0, local = 0;
      uint32_t g = 0;  // steps of this tile so far, all items (s_free / p_full / p_free phases)
      bool ok = true;
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        if (ok && !mbar_wait(bar, parity, args.err, kErrWaitMma, abort_flag)) ok = false;
        return ok;
      };
      // S(j) = Q K(j)^T into this tile's S columns
      auto issue_s = [&](int j, uint64_t qd, int qb) {
        const int idx = freq ? kvc + x : kvc + j;
        const int st = idx % kAttnKvStages;
        if (!wait(&kv_full[st], (uint32_t)(idx / kAttnKvStages) & 1)) return;
        tc_fence_after();
        const uint64_t kd = k_desc0 + (uint64_t)(st * kStep);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) mma_f16_ss(tS, qd + 2 * kk, kd + 2 * kk, idesc_qk, kk > 0 ? 1u : 0u);
        mma_commit(&s_full[x]);
        if (j == nsteps - 1) mma_commit(&q_empty[qb]);  // this tile's last read of the Q buffer
      };
      // O += P(j) V(j), P from TMEM
      auto issue_pv = [&](int j) {
        if (!wait(&p_full[x], g & 1u)) return;
        if (j == 0 && local > 0 && !wait(&o_free[x], (uint32_t)(local - 1) & 1)) return;
        tc_fence_after();
        const int idx = freq ? kvc + x : kvc + j;
        const int st = idx % kAttnKvStages;
        const uint64_t vd = v_desc0 + (uint64_t)(st * kStep);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // 16 keys per MMA: P columns kk*8.., V rows kk*16..
          mma_f16_ts(tO, tP + kk * 8, vd + kk * (2048 >> 4), idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&p_free[x]);
        mma_commit(&kv_empty[st]);  // one of the stage's readers (two in time mode)
      };
      for (int item = blockIdx.x; item < args.num_items && ok; item += gridDim.x, ++local) {
        const int qb = local & 1;
        if (!wait(&q_full[qb], (uint32_t)(local >> 1) & 1)) break;
        const uint64_t qd = q_desc0 + (uint64_t)(qb * kStep);
        // the softmax must have taken the previous S out of TMEM before S(0) overwrites it
        if (g > 0 && !wait(&s_free[x], (g - 1) & 1u)) break;
        issue_s(0, qd, qb);
        for (int j = 0; j < nsteps && ok; ++j, ++g) {
          // S(j+1) as soon as the softmax has read S(j): it runs while the exponentials of step j are made
          if (j + 1 < nsteps && wait(&s_free[x], g & 1u)) issue_s(j + 1, qd, qb);
          issue_pv(j);
        }
        kvc += kv_per_item;
      }
      mma_commit(drain);
      const uint64_t t0 = global_ns();
      while (!mbar_try_wait(drain, 0) && global_ns() - t0 < kWaitLimitNs) {
      }
    }
  }
  } else {
    if constexpr (!kFreq) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kAttnRegsHigh) : "memory");
    // ------------------------------------------------------------------ softmax + epilogue (warps 4-11)
    const int x = (warp - 4) >> 2;  // query tile of this warpgroup
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem_base + lane_off + tmem_col_s(x);
    const uint32_t tP = tmem_base + lane_off + tmem_col_p(x);
    const uint32_t tO = tmem_base + lane_off + tmem_col_o(x);
    const float kLog2e = 1.4426950408889634f;
    uint32_t g = 0;  // steps of this tile so far, all items (s_full / p_free phases)
    // This thread's query row of an item: output token, false if the row lies outside its sequence.
    auto row_token = [&](int item, long* token) -> bool {
      int seq, pos;
      if (freq) {
        seq = 4 * item + 2 * x + (r >> 6);
        pos = r & 63;
      } else {
        const int bh = item / args.q_pairs;
        seq = bh;
        pos = (item - bh * args.q_pairs) * 256 + x * 128 + r;
      }
      if (pos >= args.L || seq >= args.BH) return false;
      const int grp = seq >> 3;
      if (!freq) {  // grp = b*F + f, pos = t
        const int b = grp / args.F, f = grp - b * args.F;
        *token = (((long)b * args.T + pos) * args.F + f) * 8 + (seq & 7);
      } else {  // grp = b*T + t, pos = f
        *token = ((long)grp * args.F + pos) * 8 + (seq & 7);
      }
      return true;
    };
    // The epilogue of an item (read O, release it, scale by gate / l, store) is deferred until the next
    // item's first P has been written: the wait for the item's last O += P V then overlaps that step's
    // exponentials, and the next O = P V (which waits for o_free) starts as soon as O has been read. The
    // row's gate / l waits in shared memory; its token is recomputed from the item index.
    float* row_scale = reinterpret_cast<float*>(smem + S::kScale) + x * 128 + r;
    auto finish = [&](int prev_item) {  // 32 columns at a time (register budget of the softmax warps)
      long th;                          // token * 8 + head
      const bool valid = row_token(prev_item, &th);
      const float scale = *row_scale;
      TIn* dst = static_cast<TIn*>(args.O) + th * 64;  // [token][h*64 + d]
#pragma unroll 1
      for (int hc = 0; hc < 2; ++hc) {
        float o[32];
        tmem_ld32(tO + hc * 32, o);
        if (hc == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&o_free[x]);
        }
        if (valid) {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= scale;
          store32<TIn>(dst + hc * 32, o);
        }
      }
    };
    bool alive = true;
    for (int item = blockIdx.x; item < args.num_items && alive; item += gridDim.x) {
      // the row's gate, loaded now so the load is long done when the item ends
      long th0;
      const float gate = row_token(item, &th0) ? args.G[th0] : 0.f;
      float m_run = -INFINITY, l_run = 0.f;
      bool ok = true;
      for (int j = 0; j < nsteps; ++j, ++g) {
        if (!mbar_wait_warp(&s_full[x], g & 1u, args.err, kErrWaitSoftmax, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if constexpr (freq) {
          // a row's keys are the 64 columns of its own sequence (block quarter / 2 of the tile); the other
          // block's P is zero, and only keys < L exist. One key tile per item: no rescaling.
          const int blk = quarter >> 1;
          float sf[64];
          tmem_ld64(tS + blk * 64, sf);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s_free[x]);
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (i >= args.L) sf[i] = -INFINITY;
          float mx4[4] = {sf[0], sf[1], sf[2], sf[3]};
#pragma unroll
          for (int i = 4; i < 60; i += 8) {
            mx4[0] = fmax3(mx4[0], sf[i], sf[i + 4]);
            mx4[1] = fmax3(mx4[1], sf[i + 1], sf[i + 5]);
            mx4[2] = fmax3(mx4[2], sf[i + 2], sf[i + 6]);
            mx4[3] = fmax3(mx4[3], sf[i + 3], sf[i + 7]);
          }
          m_run = fmaxf(fmax3(mx4[0], mx4[1], sf[60]), fmax3(mx4[2], mx4[3], fmax3(sf[61], sf[62], sf[63]))) * kLog2e;
          const float2 scale2 = make_float2(kLog2e, kLog2e);
          const float2 shift2 = make_float2(-m_run, -m_run);
          float2 l2 = make_float2(0.f, 0.f);
          uint32_t pk0[16], pk1[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float2 xv = __ffma2_rn(make_float2(sf[i], sf[i + 1]), scale2, shift2);
            const float2 pv = make_float2(ex2_approx(xv.x), ex2_approx(xv.y));
            l2 = __fadd2_rn(l2, pv);
            pk0[i >> 1] = OperandType<TIn>::pack2(pv.x, pv.y);
            const float2 xw = __ffma2_rn(make_float2(sf[32 + i], sf[33 + i]), scale2, shift2);
            const float2 pw = make_float2(ex2_approx(xw.x), ex2_approx(xw.y));
            l2 = __fadd2_rn(l2, pw);
            pk1[i >> 1] = OperandType<TIn>::pack2(pw.x, pw.y);
          }
          l_run = l2.x + l2.y;
          // P and O are this tile's again once the previous item's O = P V has completed
          if (g > 0 && !mbar_wait_warp(&p_free[x], (g - 1) & 1u, args.err, kErrWaitSoftmax, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t z[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) z[i] = 0u;
          tmem_st16(tP + blk * 32, pk0);
          tmem_st16(tP + blk * 32 + 16, pk1);
          tmem_st16(tP + (1 - blk) * 32, z);
          tmem_st16(tP + (1 - blk) * 32 + 16, z);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&p_full[x]);
          if (item != (int)blockIdx.x) finish(item - gridDim.x);  // its O = P V completed: p_free above
          continue;
        }
        // the whole score row in registers (one TMEM read); the S columns are then free for the next S
        float sc[128];
        tmem_ld128(tS, sc);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[x]);
        // keys past the sequence's end -> -inf
        const int key0 = j * 128;
        const int kmax = min(128, args.L - key0);  // keys of this tile that exist
        if (kmax < 128) {
#pragma unroll
          for (int i = 0; i < 128; ++i)
            if (i >= kmax) sc[i] = -INFINITY;
        }
        float mx4[4] = {sc[0], sc[1], sc[2], sc[3]};
#pragma unroll
        for (int i = 4; i < 124; i += 8) {
          mx4[0] = fmax3(mx4[0], sc[i], sc[i + 4]);
          mx4[1] = fmax3(mx4[1], sc[i + 1], sc[i + 5]);
          mx4[2] = fmax3(mx4[2], sc[i + 2], sc[i + 6]);
          mx4[3] = fmax3(mx4[3], sc[i + 3], sc[i + 7]);
        }
        const float m_tile =
            fmaxf(fmax3(mx4[0], mx4[1], sc[124]), fmax3(mx4[2], mx4[3], fmax3(sc[125], sc[126], sc[127]))) *
            kLog2e;
        bool rescale = false;
        float alpha = 1.0f;
        if (j == 0) {
          m_run = m_tile;
        } else {
          const bool need = m_tile > m_run + kRescaleThreshold;
          rescale = __any_sync(0xffffffffu, need);
          if (need) {
            alpha = ex2_approx(m_run - m_tile);
            m_run = m_tile;
          }
        }
        // P = 2^(s log2e - m_run) as 16-bit pairs, 32 keys at a time; the last pair of every four on the
        // FMA pipe
        const float2 scale2 = make_float2(kLog2e, kLog2e);
        const float2 shift2 = make_float2(-m_run, -m_run);
        float2 l2 = make_float2(0.f, 0.f);
        auto exp_chunk = [&](int c, uint32_t(&packed)[16]) {
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const int k = c * 32 + i;
            const float2 xv = __ffma2_rn(make_float2(sc[k], sc[k + 1]), scale2, shift2);
            const float2 pv = (i & 7) == 6 ? ex2_poly2(xv) : make_float2(ex2_approx(xv.x), ex2_approx(xv.y));
            l2 = __fadd2_rn(l2, pv);
            packed[i >> 1] = OperandType<TIn>::pack2(pv.x, pv.y);
          }
        };
        {
          uint32_t packed[16];
          exp_chunk(0, packed);
          // P and O are this tile's again once the previous O += P V has completed
          if (g > 0 && !mbar_wait_warp(&p_free[x], (g - 1) & 1u, args.err, kErrWaitSoftmax, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (rescale) {  // O holds the steps < j; 16 columns at a time (register budget)
#pragma unroll 1
            for (int h = 0; h < 4; ++h) {
              float o[16];
              uint32_t u[16];
              tmem_ld16(tO + h * 16, o);
#pragma unroll
              for (int i = 0; i < 16; ++i) u[i] = __float_as_uint(o[i] * alpha);
              tmem_st16(tO + h * 16, u);
            }
          }
          tmem_st16(tP, packed);
        }
#pragma unroll
        for (int c = 1; c < 4; ++c) {
          uint32_t packed[16];
          exp_chunk(c, packed);
          tmem_st16(tP + c * 16, packed);
        }
        l_run = l_run * alpha + (l2.x + l2.y);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[x]);
        // step 0 waited (p_free) for the previous item's last O += P V and did not rescale O
        if (j == 0 && item != (int)blockIdx.x) finish(item - gridDim.x);
      }
      if (!ok) {
        alive = false;
        break;
      }
      *row_scale = gate / l_run;  // read back by this thread's deferred epilogue
    }
    // the last item: O is final once its last O += P V completed
    if (alive && (int)blockIdx.x < args.num_items &&
        mbar_wait_warp(&p_free[x], (g - 1) & 1u, args.err, kErrWaitSoftmax, abort_flag)) {
      tc_fence_after();
      finish(blockIdx.x + ((args.num_items - 1 - (int)blockIdx.x) / (int)gridDim.x) * gridDim.x);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace trc
