// Fused MLP chain with the hidden activations held in tensor memory (the A operand of the next
// layer's MMA comes straight from TMEM), for chains with one wide first layer:
//   dlrm_botmlp  apps/dlrm_botmlp/pipelined/dlrm_botmlp_pl.cuh:139-173  16/32 -> 512 -> 256 -> 128
//   bert_ffn     apps/bert_ffn/pipelined/bert_ffn_pl.cuh:132-162        128 -> 512 -> 128, + x, LN
// (and the FFN stage of apps/bert_addln_ffn).
//
// Why a third kernel family: in the weight-streaming kernel the 128 x 512 first-layer activation
// occupies 128 KB of shared memory as the next layer's A operand, which leaves two weight stages;
// the weight ring is then latency-bound (one stage per half round trip) and the tensor pipe idles
// (DLRM bottom: 18% busy, L2 9% busy). Here the activations never touch shared memory:
//
//   TMEM columns [0, 256)    S: accumulators. The first layer runs as 128-column chunks that
//                            alternate between S[0, 128) and S[128, 256); later layers
//                            (N <= 256) accumulate at S[0, N).
//   TMEM columns [256, 512)  A: the previous layer's activation as packed 16-bit pairs
//                            (N <= 512 values per row), read by TS-form tcgen05.mma.
//
// so shared memory holds only the resident x tile (double-buffered), biases, output staging and a
// weight ring of up to eight 32 KB stages.
//
//   warp 0      TMA producer: x tiles, then every layer's weights as stages of up to 64 rows x
//               all N columns (the first layer per 128-column chunk), L2-resident.
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer.
//   warps 2-9   epilogue, two warps per TMEM lane quarter: thread t of a quarter owns row t of
//               the tile; warp group 0 handles the first half of each accumulator's columns,
//               group 1 the second half.
//
// Hand-offs (every wait bounded): acc_full[2] (a job's MMAs are complete, jobs alternate),
// s_free[2] (the epilogue has read S half h), act_ready (the next layer's A operand is written),
// b_full / b_empty (weight ring), x_full / x_empty (x tiles).
#pragma once

#include "chain_common.cuh"
#include "gp_ptx.cuh"
#include "mlp_resident.cuh"

namespace gp {

template <class C, int CG = 1>
struct TmemLayout {
  static constexpr int NL = C::NL;
  static constexpr int K0 = C::K(0);
  static constexpr int N0 = C::N(0);
  static constexpr int NLast = C::N(NL - 1);
  static_assert(NL >= 2 && NL <= kMaxLayers, "two or more layers");
  static_assert(K0 % 16 == 0 && K0 <= 128, "resident x tile: at most two 64-column panels");
  static_assert(N0 % 128 == 0 && N0 <= 512, "first layer: 128-column chunks, at most 512 columns");
  __host__ __device__ static constexpr bool laterOk() {
    for (int l = 1; l < NL; ++l) {
      if (C::K(l) != C::N(l - 1)) return false;
      if (C::N(l) % 64 != 0 || C::N(l) > 256) return false;
    }
    return true;
  }
  static_assert(laterOk(), "layers >= 1: K = previous N, N a multiple of 64 up to 256");
  __host__ __device__ static constexpr bool pairOk() {
    for (int l = 1; l < NL; ++l)
      if (C::N(l) % 128 != 0) return false;
    return true;
  }
  static_assert(CG == 1 || (CG == 2 && pairOk()), "CTA pairs stage half of every N: N a multiple of 128");
  static constexpr bool kLN = C::TAIL == kTailLayerNorm || C::TAIL == kTailResidualLN;
  static constexpr bool kResid = C::TAIL == kTailResidualLN;
  static_assert(!kResid || K0 == NLast, "residual tail: the residual is x itself");
  static constexpr int kXPanels = (K0 + kPanel - 1) / kPanel;
  static constexpr int kChunks0 = N0 / 128;
  static constexpr int kBK0 = K0 < 64 ? K0 : 64;  // first-layer stage rows
  static constexpr int kBK = 64;                  // later-layer stage rows
  __host__ __device__ static constexpr int maxLaterN() {
    int m = 64;
    for (int l = 1; l < NL; ++l) m = C::N(l) > m ? C::N(l) : m;
    return m;
  }
  __host__ __device__ static constexpr int biasFloats() {
    int s = 0;
    for (int l = 0; l < NL; ++l) s += C::N(l);
    return s;
  }
  __host__ __device__ static constexpr int biasOff(int l) {
    int s = 0;
    for (int i = 0; i < l; ++i) s += C::N(i);
    return s;
  }
  // bytes of one stage in this CTA (a CTA pair stages half of the columns in each CTA)
  static constexpr int kStageBytesMax =
      ((kBK * maxLaterN() * 2 > kBK0 * 128 * 2) ? kBK * maxLaterN() * 2 : kBK0 * 128 * 2) / CG;
  static constexpr int kXBytes = kXPanels * kPanelBytes;  // one x slot
  static constexpr int kEpiWarps = 8;
  static constexpr int kStgBytes = kEpiWarps * 2 * 2048;  // two 32 x 32 output tiles per warp
  static constexpr int kBiasBytes = ((biasFloats() * 4 + 1023) / 1024) * 1024;
  static constexpr int kLnBytes = kLN ? 2 * NLast * 4 : 0;
  static constexpr int kXchgBytes = kLN ? 2 * kBM * 8 : 0;
  static constexpr int kBarBytes = 512;
  static constexpr int kOffX = 0;
  static constexpr int kOffB = kOffX + 2 * kXBytes;
  static constexpr int kFixed = 2 * kXBytes + kStgBytes + kBiasBytes + kLnBytes + kXchgBytes + kBarBytes;
  static constexpr int kBStagesRaw = (kSmemLimit - kFixed) / kStageBytesMax;
  static constexpr int kBStages = kBStagesRaw > 8 ? 8 : kBStagesRaw;
  static_assert(kBStages >= 2, "shared memory budget");
  static constexpr int kOffStg = kOffB + kBStages * kStageBytesMax;
  static constexpr int kOffBias = kOffStg + kStgBytes;
  static constexpr int kOffLn = kOffBias + kBiasBytes;
  static constexpr int kOffXchg = kOffLn + kLnBytes;
  static constexpr int kOffBar = kOffXchg + kXchgBytes;
  static constexpr int kSmemBytes = kOffBar + kBarBytes;
  static_assert(kSmemBytes <= kSmemLimit, "shared memory budget");
  static_assert(kOffB % 1024 == 0 && kStageBytesMax % 1024 == 0 && kOffStg % 1024 == 0, "alignment");
  static constexpr int kUnitRows = kBM * CG;
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr uint32_t kACol = 256;  // TMEM column of the packed activation
};

template <class C, int CG>
__device__ __forceinline__ void mlp_tmem_body(const TensorMaps& tm, const ChainArgs& args) {
  using T = typename C::T;
  using L = TmemLayout<C, CG>;
  constexpr bool kPair = CG == 2;
  using H = typename std::conditional<C::HIDDEN_F16, __half, T>::type;  // hidden activation type
  constexpr int NL = C::NL;
  constexpr int kBS = L::kBStages;

  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* b_full = bars;          // [8]
  uint64_t* b_empty = bars + 8;     // [8]
  uint64_t* x_full = bars + 16;     // [2]
  uint64_t* x_empty = bars + 18;    // [2]
  uint64_t* acc_full = bars + 20;   // [2]  by job parity
  uint64_t* s_free = bars + 22;     // [2]  by S half
  uint64_t* act_ready = bars + 24;  // [1]
  uint64_t* mma_done = bars + 25;   // [1]
  uint64_t* pair_bar = bars + 26;   // [4]  the two epilogue warps of each TMEM lane quarter
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 30);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 31);
  float* bias_s = reinterpret_cast<float*>(smem + L::kOffBias);
  float* ln_g = reinterpret_cast<float*>(smem + L::kOffLn);
  float* ln_b = ln_g + L::NLast;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_units = args.num_tiles;  // in units of kUnitRows rows
  const uint32_t rank = kPair ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int unit0 = kPair ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int units_step = kPair ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  if ((smem_u32(smem) & 1023u) != 0) {
    pdl_wait_prior();
    if (threadIdx.x == 0) atomicCAS(args.status, 0, kDevBadSmemAlign);
    return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < 8; ++s) {
      mbar_init(smem_u32(&b_full[s]), 1);
      mbar_init(smem_u32(&b_empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&x_full[s]), 1);
      // the residual tail reads x in the epilogue: then this CTA's epilogue warps release the
      // slot; otherwise the (pair leader's) MMA commit does
      mbar_init(smem_u32(&x_empty[s]), L::kResid ? L::kEpiWarps : 1);
      mbar_init(smem_u32(&acc_full[s]), 1);
      mbar_init(smem_u32(&s_free[s]), L::kEpiWarps * CG);  // the leader's count both CTAs
    }
    mbar_init(smem_u32(act_ready), L::kEpiWarps * CG);
    mbar_init(smem_u32(mma_done), 1);
    for (int i = 0; i < 4; ++i) mbar_init(smem_u32(&pair_bar[i]), 64);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm.x);
    prefetch_tmap(&tm.out);
  }
  // Everything above overlaps the previous kernel of the stream. Global memory is touched only
  // after griddepcontrol.wait, except the per-column parameters when the launch marked them safe
  // (pdl_early bit 1), which are staged first.
  const int early = args.pdl_early;
  if ((early & 1) == 0) pdl_wait_prior();
  for (int l = 0; l < NL; ++l) {
    const T* b = reinterpret_cast<const T*>(args.bias[l]);
    for (int i = threadIdx.x; i < C::N(l); i += blockDim.x)
      bias_s[L::biasOff(l) + i] = b != nullptr ? Elem<T>::to_f(b[i]) : 0.0f;
  }
  if constexpr (L::kLN) {
    const T* g = reinterpret_cast<const T*>(args.gamma);
    const T* b = reinterpret_cast<const T*>(args.beta);
    for (int i = threadIdx.x; i < L::NLast; i += blockDim.x) {
      ln_g[i] = g != nullptr ? Elem<T>::to_f(g[i]) : 1.0f;
      ln_b[i] = b != nullptr ? Elem<T>::to_f(b[i]) : 0.0f;
    }
  }
  if (early & 1) pdl_wait_prior();
  if (threadIdx.x == 0) pdl_launch_dependents();  // after this grid's wait: only this grid can precede the next one
  if (warp == 1) {
    if constexpr (kPair) {
      tmem_alloc_pair(smem_u32(tmem_holder), 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(tmem_holder), 512);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (kPair) {
    cluster_sync_all();  // the peer's barriers are initialised before any remote arrival
  } else {
    __syncthreads();
  }
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const WaitCtx wctx{args.status, abort_flag, args.timeout_ns};
  // barrier address as seen by the loads / arrivals of this CTA (the leader's in a pair)
  auto leader_bar = [&](const uint64_t* b) -> uint32_t {
    return kPair ? mapa_shared(smem_u32(b), 0) : smem_u32(b);
  };
  auto commit_any = [&](uint64_t* bar) {
    if constexpr (kPair) mma_commit_pair(smem_u32(bar), 0x3); else mma_commit(smem_u32(bar));
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      const uint64_t keep = l2_policy_evict_last();
      const uint64_t stream = l2_policy_evict_first();
      int bs = 0, xs = 0;
      uint32_t bph = 0, xph = 0;
      bool ok = true;
      // bytes: the whole stage (both CTAs of a pair); this CTA loads its half of the columns
      auto stage = [&](const CUtensorMap* map, int row, int blk, uint32_t bytes) -> bool {
        if (!mbar_wait<kPair>(smem_u32(&b_empty[bs]), bph ^ 1, wctx, kDevTimeoutProducer)) return false;
        if (leader) mbar_arrive_expect_tx(smem_u32(&b_full[bs]), bytes);
        const uint32_t dst = smem_u32(smem + L::kOffB + bs * L::kStageBytesMax);
        if constexpr (kPair) {
          tma_load_3d_pair(dst, map, leader_bar(&b_full[bs]), 0, row, blk, keep);
        } else {
          tma_load_3d_hint(dst, map, smem_u32(&b_full[bs]), 0, row, blk, keep);
        }
        if (++bs == kBS) { bs = 0; bph ^= 1; }
        return true;
      };
#pragma unroll 1
      for (int unit = unit0; ok && unit < num_units; unit += units_step) {
        const int row_base = unit * L::kUnitRows + static_cast<int>(rank) * kBM;
        if (!mbar_wait<kPair>(smem_u32(&x_empty[xs]), xph ^ 1, wctx, kDevTimeoutProducer)) break;
        if (args.inject != 1) {
          if (leader) mbar_arrive_expect_tx(smem_u32(&x_full[xs]), L::kXBytes * CG);
          for (int p = 0; p < L::kXPanels; ++p) {
            const uint32_t dst = smem_u32(smem + L::kOffX + xs * L::kXBytes + p * kPanelBytes);
            if constexpr (kPair) {
              tma_load_2d_pair(dst, &tm.x, leader_bar(&x_full[xs]), p * kPanel, row_base, stream);
            } else {
              tma_load_2d_hint(dst, &tm.x, smem_u32(&x_full[xs]), p * kPanel, row_base, stream);
            }
          }
        }
        if (++xs == 2) { xs = 0; xph ^= 1; }
        // first layer: per 128-column chunk, kBK0-row stages of two 64-column blocks (one per
        // CTA of a pair)
        for (int j = 0; ok && j < L::kChunks0; ++j)
          for (int r0 = 0; ok && r0 < L::K0; r0 += L::kBK0)
            ok = stage(&tm.w[0], r0, 2 * j + static_cast<int>(rank), L::kBK0 * 128 * 2);
        for (int l = 1; ok && l < NL; ++l)
          for (int r0 = 0; ok && r0 < C::K(l); r0 += L::kBK)
            ok = stage(&tm.w[l], r0, static_cast<int>(rank) * (C::N(l) / CG / 64), L::kBK * C::N(l) * 2);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0 && leader) {
      const uint32_t b_sm = smem_u32(smem + L::kOffB);
      const uint32_t x_sm = smem_u32(smem + L::kOffX);
      int bs = 0, xs = 0;
      uint32_t bph = 0, xph = 0, aph = 0;
      uint32_t sph[2] = {0, 0};
      int job = 0;
      bool ok = true;
      auto take_s = [&](int h) -> bool {  // S half h is free (the epilogue has read it)
        if (!mbar_wait<kPair>(smem_u32(&s_free[h]), sph[h] ^ 1, wctx, kDevTimeoutMma)) return false;
        sph[h] ^= 1;
        return true;
      };
      auto mma_ss_any = [&](uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
        if constexpr (kPair) mma_ss_pair(d, a, b, idesc, acc); else mma_ss(d, a, b, idesc, acc);
      };
      auto mma_ts_any = [&](uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
        if constexpr (kPair) mma_ts_pair(d, a, b, idesc, acc); else mma_ts(d, a, b, idesc, acc);
      };
      constexpr uint32_t kIdesc0 = make_idesc_f16(L::kUnitRows, 128, Elem<T>::kIsBf16, 0, 1);
#pragma unroll 1
      for (int unit = unit0; ok && unit < num_units; unit += units_step) {
        const int xcur = xs;
        if (!mbar_wait<kPair>(smem_u32(&x_full[xcur]), xph, wctx, kDevTimeoutMma)) break;
        tc_fence_after();
        // first layer: SS MMAs (x panels x W0 chunk stages) into alternating S halves
#pragma unroll 1
        for (int j = 0; ok && j < L::kChunks0; ++j) {
          const int h = j & 1;
          if (!take_s(h)) { ok = false; break; }
          tc_fence_after();
#pragma unroll 1
          for (int r0 = 0; r0 < L::K0; r0 += L::kBK0) {
            if (!mbar_wait<kPair>(smem_u32(&b_full[bs]), bph, wctx, kDevTimeoutMma)) { ok = false; break; }
            tc_fence_after();
            const uint32_t bst = b_sm + bs * L::kStageBytesMax;
            const uint32_t xp = x_sm + xcur * L::kXBytes + (r0 / kPanel) * kPanelBytes;
            for (int k = 0; k < L::kBK0 / 16; ++k) {
              const uint64_t adesc = make_sdesc_sw128(xp + ((r0 % kPanel) / 16 + k) * 32, 16, 1024);
              const uint64_t bdesc = make_sdesc_sw128(bst + k * 2048, L::kBK0 * 128, 1024);
              mma_ss_any(tmem_base + h * 128, adesc, bdesc, kIdesc0, (r0 | k) != 0 ? 1u : 0u);
            }
            commit_any(&b_empty[bs]);
            if (++bs == kBS) { bs = 0; bph ^= 1; }
          }
          if (!ok) break;
          commit_any(&acc_full[job & 1]);
          ++job;
        }
        if (!ok) break;
        if constexpr (!L::kResid) commit_any(&x_empty[xcur]);  // x is read by layer 0 only
        // later layers: TS MMAs, A = the packed activation in TMEM columns [256, ...)
#pragma unroll 1
        for (int l = 1; ok && l < NL; ++l) {
          if (!mbar_wait<kPair>(smem_u32(act_ready), aph, wctx, kDevTimeoutMma)) { ok = false; break; }
          aph ^= 1;
          if (!take_s(0) || (C::N(l) > 128 && !take_s(1))) { ok = false; break; }
          tc_fence_after();
          const uint32_t idesc = make_idesc_f16(L::kUnitRows, C::N(l), (C::HIDDEN_F16 ? 0 : Elem<T>::kIsBf16), 0, 1);
#pragma unroll 1
          for (int r0 = 0; r0 < C::K(l); r0 += L::kBK) {
            if (!mbar_wait<kPair>(smem_u32(&b_full[bs]), bph, wctx, kDevTimeoutMma)) { ok = false; break; }
            tc_fence_after();
            const uint32_t bst = b_sm + bs * L::kStageBytesMax;
            for (int k = 0; k < L::kBK / 16; ++k) {
              const uint64_t bdesc = make_sdesc_sw128(bst + k * 2048, L::kBK * 128, 1024);
              mma_ts_any(tmem_base, tmem_base + L::kACol + (r0 / 16 + k) * 8, bdesc, idesc, (r0 | k) != 0 ? 1u : 0u);
            }
            commit_any(&b_empty[bs]);
            if (++bs == kBS) { bs = 0; bph ^= 1; }
          }
          if (!ok) break;
          commit_any(&acc_full[job & 1]);
          ++job;
        }
        if (++xs == 2) { xs = 0; xph ^= 1; }
      }
      commit_any(mma_done);  // every issued MMA has completed before TMEM is released
    }
    if (lane == 0) {
      volatile int no_abort = 0;
      WaitCtx drain{args.status, &no_abort, args.timeout_ns};
      mbar_wait<kPair>(smem_u32(mma_done), 0, drain, kDevTimeoutMma);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..9)
    const int q = warp & 3;          // TMEM lane quarter
    const int eg = (warp - 2) >> 2;  // column half of each accumulator handled by this warp
    const int r = q * 32 + lane;     // row within the tile
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    uint8_t* stg = smem + L::kOffStg + (warp - 2) * 4096;
    float* xchg = reinterpret_cast<float*>(smem + L::kOffXchg);
    uint32_t acc_ph[2] = {0, 0};
    uint32_t pph = 0;
    int job = 0, sb = 0, xs = 0;
    bool ok = true;
    auto wait_job = [&]() -> bool {
      const int i = job & 1;
      if (!mbar_wait<kPair>(smem_u32(&acc_full[i]), acc_ph[i], wctx, kDevTimeoutEpilogue)) return false;
      acc_ph[i] ^= 1;
      ++job;
      tc_fence_after();
      return true;
    };
    // a hand-off the (pair leader's) MMA issuer waits on
    auto arrive = [&](uint64_t* bar) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (kPair) mbar_arrive_cluster(leader_bar(bar)); else mbar_arrive(smem_u32(bar));
      }
    };
    // a hand-off to this CTA's own producer
    auto arrive_local = [&](uint64_t* bar) {
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(bar));
    };
    auto pair_sync = [&]() -> bool {
      mbar_arrive(smem_u32(&pair_bar[q]));
      const bool ok2 = mbar_wait(smem_u32(&pair_bar[q]), pph, wctx, kDevTimeoutEpilogue);
      pph ^= 1;
      return ok2;
    };
    // bias + activation of 32 accumulator columns, packed to 16 hidden-type pairs
    auto hidden32 = [&](const uint32_t (&v)[32], const float* bl, int act_id, uint32_t (&pk)[16]) {
      act_dispatch(act_id, [&](auto actc) {
        constexpr int A = decltype(actc)::value;
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pk[i] = Elem<H>::pack(act_t<A>(__uint_as_float(v[2 * i]) + bl[2 * i]),
                                act_t<A>(__uint_as_float(v[2 * i + 1]) + bl[2 * i + 1]));
      });
    };
#pragma unroll 1
    for (int unit = unit0; ok && unit < num_units; unit += units_step) {
      const int row0 = unit * L::kUnitRows + static_cast<int>(rank) * kBM + q * 32;
      // ---- first layer: each warp converts 64 columns of every 128-column chunk
#pragma unroll 1
      for (int j = 0; ok && j < L::kChunks0; ++j) {
        if (!wait_job()) { ok = false; break; }
        const int h = j & 1;
        uint32_t v[2][32];
        tmem_ld32(t_lane + h * 128 + eg * 64, v[0]);
        tmem_ld32(t_lane + h * 128 + eg * 64 + 32, v[1]);
        tmem_wait_ld();
        const float* bl = bias_s + j * 128 + eg * 64;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t pk[16];
          hidden32(v[c], bl + c * 32, C::ACT(0), pk);
          tmem_st16(t_lane + L::kACol + (j * 128 + eg * 64 + c * 32) / 2, pk);
        }
        tmem_wait_st();
        arrive(&s_free[h]);
      }
      if (!ok) break;
      arrive(act_ready);
      // ---- hidden layers >= 1: this warp's half of the columns, back into the A region
#pragma unroll 1
      for (int l = 1; ok && l + 1 < NL; ++l) {
        if (!wait_job()) { ok = false; break; }
        const int half = C::N(l) / 2;
        const float* bl = bias_s + L::biasOff(l) + eg * half;
#pragma unroll 1
        for (int c = 0; c < half / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(t_lane + eg * half + c * 32, v);
          tmem_wait_ld();
          uint32_t pk[16];
          hidden32(v, bl + c * 32, C::ACT(l), pk);
          tmem_st16(t_lane + L::kACol + (eg * half + c * 32) / 2, pk);
        }
        tmem_wait_st();
        arrive(&s_free[0]);
        if (C::N(l) > 128) arrive(&s_free[1]);
        arrive(act_ready);
      }
      if (!ok) break;
      // ---- last layer: activation or (residual +) LayerNorm, stored through staging with TMA
      if (!wait_job()) { ok = false; break; }
      constexpr int NLast = L::NLast;
      constexpr int half = NLast / 2;
      const float* bl = bias_s + L::biasOff(NL - 1) + eg * half;
      const uint8_t* xt = smem + L::kOffX + xs * L::kXBytes;
      // residual (x, from the resident tile in shared memory: SW128 K-major panels)
      auto resid_add = [&](int col0, float (&y)[32]) {
        if constexpr (L::kResid) {
          const uint8_t* line = xt + (col0 / kPanel) * kPanelBytes + r * 128;
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const int chunk = ((col0 % kPanel) / 8) + jj;
            const uint4 w = *reinterpret_cast<const uint4*>(line + ((chunk ^ (r & 7)) * 16));
            const T* t = reinterpret_cast<const T*>(&w);
#pragma unroll
            for (int e = 0; e < 8; ++e) y[jj * 8 + e] += Elem<T>::to_f(t[e]);
          }
        }
      };
      float mean = 0.f, rstd = 1.f;
      if constexpr (L::kLN) {
        // shifted sums per warp half, combined across the pair (parallel variance)
        float s = 0.f, sq = 0.f, k = 0.f;
#pragma unroll 1
        for (int c = 0; c < half / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(t_lane + eg * half + c * 32, v);
          tmem_wait_ld();
          float y[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) y[i] = __uint_as_float(v[i]) + bl[c * 32 + i];
          resid_add(eg * half + c * 32, y);
          if (c == 0) k = y[0];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float d = y[i] - k;
            s += d;
            sq = fmaf(d, d, sq);
          }
        }
        const float n_h = static_cast<float>(half);
        const float mean_me = k + s / n_h;
        const float m2_me = fmaxf(sq - s * (s / n_h), 0.0f);
        float2* xsx = reinterpret_cast<float2*>(xchg);
        xsx[eg * kBM + r] = make_float2(mean_me, m2_me);
        if (!pair_sync()) { ok = false; break; }
        const float2 other = xsx[(eg ^ 1) * kBM + r];
        if (!pair_sync()) { ok = false; break; }
        const float2 h0 = eg == 0 ? make_float2(mean_me, m2_me) : other;
        const float2 h1 = eg == 0 ? other : make_float2(mean_me, m2_me);
        mean = 0.5f * (h0.x + h1.x);
        const float delta = h1.x - h0.x;
        const float var = (h0.y + h1.y + delta * delta * (0.5f * n_h)) * (1.0f / NLast);
        rstd = rsqrtf(var + args.ln_eps);
      }
#pragma unroll 1
      for (int c = 0; c < half / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(t_lane + eg * half + c * 32, v);
        tmem_wait_ld();
        float y[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) y[i] = __uint_as_float(v[i]) + bl[c * 32 + i];
        resid_add(eg * half + c * 32, y);
        uint32_t pk[16];
        if constexpr (L::kLN) {
          const int col = eg * half + c * 32;
#pragma unroll
          for (int i = 0; i < 16; ++i)
            pk[i] = Elem<T>::pack((y[2 * i] - mean) * rstd * ln_g[col + 2 * i] + ln_b[col + 2 * i],
                                  (y[2 * i + 1] - mean) * rstd * ln_g[col + 2 * i + 1] + ln_b[col + 2 * i + 1]);
        } else {
          act_dispatch(C::ACT(NL - 1), [&](auto actc) {
            constexpr int A = decltype(actc)::value;
#pragma unroll
            for (int i = 0; i < 16; ++i) pk[i] = Elem<T>::pack(act_t<A>(y[2 * i]), act_t<A>(y[2 * i + 1]));
          });
        }
        if (c + 1 == half / 32) {
          // every accumulator column of this warp is read: S may take the next tile's chunks
          arrive(&s_free[0]);
          if (NLast > 128) arrive(&s_free[1]);
          if constexpr (L::kResid) arrive_local(&x_empty[xs]);
        }
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
        stage_chunk32(stg + sb * 2048, lane, pk);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (row0 < args.m) tma_store_2d(&tm.out, smem_u32(stg + sb * 2048), eg * half + c * 32, row0);
          bulk_commit_group();
        }
        sb ^= 1;
      }
      if (++xs == 2) xs = 0;
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }
  tc_fence_before();
  if constexpr (kPair) {
    cluster_sync_all();  // no CTA leaves while the pair's MMAs may still read its memory
  } else {
    __syncthreads();
  }
  if (warp == 1) {
    tc_fence_after();
    if constexpr (kPair) tmem_dealloc_pair(tmem_base, 512); else tmem_dealloc(tmem_base, 512);
  }
}

template <class C>
__global__ void __launch_bounds__(320, 1)
    mlp_tmem_kernel(const __grid_constant__ TensorMaps tm, const ChainArgs args) {
  mlp_tmem_body<C, 1>(tm, args);
}

// CTA-pair form: 256-row units, 256-row MMAs issued by the leader over both CTAs' TMEM
// activations, each CTA staging half of the columns of every weight stage.
template <class C>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(320, 1)
    mlp_tmem_pair_kernel(const __grid_constant__ TensorMaps tm, const ChainArgs args) {
  mlp_tmem_body<C, 2>(tm, args);
}

}  // namespace gp
