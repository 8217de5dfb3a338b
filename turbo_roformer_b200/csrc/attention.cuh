// Frequency-mode attention (sequences over the bands of one frame and head) on tcgen05, and what the
// time-mode kernel (attention_time.cuh) shares with it: the argument block, the TMEM/shared layouts'
// helpers, the FMA-pipe exponential and the rescale threshold.
//
// Replaces the reference's AVX-512 `attention` kernel for mode 1 (LoggeL/turbo-roformer
// src/turbo_roformer/csrc/kernels.cpp:255-388): per (sequence, head) S = Q K^T (scale folded into W_q),
// softmax over the keys, O = P V, then x sigmoid gate, head merge and scatter back to token order.
// Sequences are L = bands <= 64 long, so one 128-row query tile holds two sequences (block-diagonal
// mask: a row reads only the 64 score columns of its own sequence) and has a single 128-key tile:
//   * S = Q K^T (both operands in shared memory) lands in TMEM; the softmax warps read their row's 64
//     scores, write 16-bit P to its own TMEM columns (zeros for the other sequence's keys), and the tensor
//     core computes O = P V with P read straight from TMEM. One key tile per item: no rescaling.
//   * A CTA owns two query tiles (A, B), each with its own key stage and MMA-issuing thread (warps 1, 2);
//     an item is four sequences (two per tile). Persistent CTAs; Q double buffered; each item's epilogue
//     (gate / l, store) is deferred to the next item's step, after its P is written.
// Layout: Q, K, V are [BH, L, 64] 16-bit, row-major, unpadded; the 3-D TMA maps (box 64 rows x 2
// sequences) zero-fill rows >= L.
// Roles (384 threads): warp 0 TMA, warp 1 MMA issuer of tile A + TMEM owner, warp 2 MMA issuer of tile B,
// warp 3 idle; warps 4-7 softmax + epilogue of tile A, warps 8-11 of tile B (thread = query row; warp w
// reads TMEM lanes 32 (w % 4) ..).
#pragma once

#include "gemm.cuh"  // store32
#include "sm100.cuh"

namespace trc {

constexpr int kAttnThreads = 384;
// Key/value stages. Frequency mode loads one stage per tile and item (tile A, tile B, tile A, ...): with an
// even stage count, stage (2 item + tile) % kAttnKvStages is only ever used by that one tile, so each
// tile's MMA issuer waits on every phase of its stages in order. With an odd count the tiles would share
// stages, and a tile running an item ahead could wait on a stage whose previous phase (the other tile's
// load) had not completed yet, where a parity wait cannot tell the two phases apart.
constexpr int kAttnKvStages = 4;
static_assert(kAttnKvStages % 2 == 0, "frequency mode needs per-tile stages");

struct AttnArgs {
  int num_items;  // work items
  int q_pairs;    // time: items (groups of three 128-row query tiles) per sequence
  int n_kv;       // time: 64-key steps per item
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

template <typename TIn>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attention_freq_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
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
  constexpr int nsteps = 1;       // key tiles per query tile and item
  constexpr int kv_per_item = 2;  // key/value loads per item (one per tile)

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
      mbar_init(&kv_empty[s], 1);  // each stage holds one tile's keys
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
  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int kvc = 0, local = 0, q_issued = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < args.num_items && ok; item += gridDim.x, ++local) {
        const int bh = 4 * item;  // first of the item's four sequences
        const int qb = local & 1;
        if (!mbar_wait(&q_empty[qb], ((uint32_t)(local >> 1) & 1) ^ 1, args.err, kErrWaitProducer, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&q_full[qb], 2 * S::kTile);
        uint8_t* qbuf = smem + S::kQ + qb * 2 * S::kTile;
        tma_load_3d(qbuf, &map_q, &q_full[qb], 0, 0, bh);
        tma_load_3d(qbuf + S::kTile, &map_q, &q_full[qb], 0, 0, bh + 2);
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
          tma_load_3d(kb, &map_k, &kv_full[st], 0, 0, bh + 2 * j);
          tma_load_3d(kb + S::kTile, &map_v, &kv_full[st], 0, 0, bh + 2 * j);
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
        const int idx = kvc + x;  // tile x's own key stage
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
        const int idx = kvc + x;  // tile x's own key stage
        const int st = idx % kAttnKvStages;
        const uint64_t vd = v_desc0 + (uint64_t)(st * kStep);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // 16 keys per MMA: P columns kk*8.., V rows kk*16..
          mma_f16_ts(tO, tP + kk * 8, vd + kk * (2048 >> 4), idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&p_free[x]);
        mma_commit(&kv_empty[st]);
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
      const int seq = 4 * item + 2 * x + (r >> 6);
      const int pos = r & 63;
      if (pos >= args.L || seq >= args.BH) return false;
      const int grp = seq >> 3;  // grp = b*T + t, pos = f
      *token = ((long)grp * args.F + pos) * 8 + (seq & 7);
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
