// A chain of wide layers as ONE persistent tcgen05 kernel, for the chains whose hidden
// activations are too wide for one SM (BERT-large FFN 1024 -> 4096 -> 1024 + x, LayerNorm; DLRM
// top 480 -> 1024 -> 1024 -> 512 -> 256 -> 1 sigmoid).
//
// The reference runs such chains as pipeline stages joined by L2-resident queues
// (apps/bert_ffn/pipelined/bert_ffn_pl.cuh:82-95, apps/dlrm_topmlp/pipelined/dlrm_topmlp_pl.cuh:
// 185-224). Here every CTA pair runs the same warp-specialised GEMM roles as mlp_gemm.cuh (TMA
// producer, cta_group::2 MMA issuer, eight epilogue warps) over a single tile sequence that mixes
// all layers of the chain:
//
//   step i:  layer 0 tiles of row block i, layer 1 tiles of row block i - lag_1, ...,
//            then (LayerNorm chains) the LayerNorm tile of row block i - lag_ln
//
// A row block is 256 rows; a layer tile is 256 rows x 256 output columns. A pair claims the next
// position of the sequence (a global counter) whenever its producer is ready for another tile, and
// hands the position to its MMA issuer, its epilogue warps and the other CTA of the pair through a
// small ring of tile ids in shared memory (claiming in order balances the layers' different tile
// durations; a fixed position-to-pair assignment measured ~1.5x the ideal time in a simulation of
// the schedule). Each layer's output goes to a ring of row blocks in global memory, reused every
// ring_q row blocks (the intermediates are read back soon after they are written, instead of
// living in full-size buffers); the last layer writes the final rows (or, for LayerNorm chains,
// an fp32 ring that the LayerNorm tiles read). Completion counters per (layer, row block) order the tiles:
//
//   read after write   a layer-l tile's producer waits until all layer-(l-1) tiles of its row
//                      block have stored their rows (each epilogue warp adds 1 after its stores
//                      complete: 16 per tile of a pair);
//   write after read   an epilogue waits, before overwriting a ring slot, until the consumers of
//                      the row block that held it (layer l+1 tiles, or the LayerNorm tile) are done.
//
// Every dependency points to an earlier position of the sequence (lags >= 1, rings deeper than
// the lags), positions are claimed in order and every pair works through its claims in order, and
// all CTAs are resident (persistent grid of at most the co-resident clusters), so the lowest
// unfinished claimed tile can always progress. Every wait is bounded and reports through the
// status word.
#pragma once

#include "mlp_gemm.cuh"

namespace gp {

constexpr int kChainMaxStages = 4;
constexpr int kDevTimeoutDependency = 0x700;  // a wait on another tile's completion counter ran out
constexpr int kDevBadSchedule = 0x800;        // a decoded tile outside the chain (no memory touched)

struct ChainStageArgs {
  int n, k, n_tiles;  // layer width N, input width K, N / 256
  int act;            // activation after bias (+ residual)
  int out_kind;       // 0: 16-bit rows by TMA; 1: fp32 rows by TMA; 2: sigmoid head, one 16-bit value per row
  int ring_q;         // row blocks in this layer's output ring; 0: output rows indexed by row (final)
  int a_bf16;         // operand type of this layer's MMAs (A and B): bf16, else fp16
  int out_bf16;       // 16-bit output type
  int lag;            // schedule step of this layer's row block 0
  int bias_off;       // offset of this layer's bias in the staged fp32 bias array
  const void* bias;   // [n] 16-bit, or null
  int bias_bf16;
  const void* resid;  // [m, n] 16-bit rows added before the activation, or null
  int resid_bf16;
};

struct GemmChainArgs {
  int m;
  int n_blocks;  // ceil(m / 256)
  int n_stages;
  int total;     // positions in the tile sequence
  int n_steps;   // steps of the sequence (the largest lag + n_blocks)
  ChainStageArgs st[kChainMaxStages];
  int* counters;   // [(n_stages + 1) * n_blocks], zero at launch
  int* next_tile;  // claim counter of the tile sequence, zero at launch
  // LayerNorm tiles (ln != 0): over the last layer's fp32 ring, rows [m, ln_n] into `out`
  int ln, ln_lag, ln_n;
  const float* ln_ring;
  const void* gamma;
  const void* beta;
  int g_bf16;
  float ln_eps;
  void* out;  // final rows (LayerNorm output, or the sigmoid head's [m, 1])
  int out_bf16;
  const void* head_w;  // sigmoid head [N_last] 16-bit, and its bias [1]
  const void* head_b;
  int bias_total;  // staged bias floats (sum of the layers' n)
  int* status;
  unsigned long long timeout_ns;
  int inject;  // fault injection 1: completion signals are dropped, so dependency waits run out
};

struct GemmChainMaps {
  CUtensorMap a[kChainMaxStages];    // layer 0: x; layer l: the ring of layer l - 1
  CUtensorMap w[kChainMaxStages];    // [K, N] weights, 3-D (each CTA of a pair: half the columns)
  CUtensorMap out[kChainMaxStages];  // this layer's ring (or final rows)
};

struct GemmChainLayout {
  static constexpr int kBN = 256;
  static constexpr int kStages = 5;
  static constexpr int kABytes = kPanelBytes;             // 128 x 64 x 2
  static constexpr int kBBytes = kPanel * kBN * 2 / 2;    // 64 x 128 x 2 per CTA
  static constexpr int kStageBytes = kABytes + kBBytes;   // 32 KB per CTA
  static constexpr int kMaxBias = 5120;                   // sum of the layers' widths
  static constexpr int kMaxHead = 256;
  static constexpr int kEpiWarps = 8;
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr int kStgWarpBytes = 4096;
  static constexpr int kOffBias = kStages * kStageBytes;
  static constexpr int kOffHead = kOffBias + kMaxBias * 4;
  static constexpr int kOffStg = ((kOffHead + (kMaxHead + 4) * 4 + 1023) / 1024) * 1024;
  static constexpr int kOffBar = kOffStg + kEpiWarps * kStgWarpBytes;
  static constexpr int kBarBytes = 512;  // 32 barrier slots + the tile-id ring
  static constexpr int kTidSlots = 4;
  static constexpr int kSmemBytes = kOffBar + kBarBytes;
  static_assert(kSmemBytes <= kSmemLimit, "shared memory budget");
  static_assert(kThreads == 320, "launch bounds of mlp_gemm_chain_kernel");
};

// ------------------------------------------------------------------------------------------ schedule
// tiles of step i (layers in order, then the LayerNorm tile)
__device__ __forceinline__ int chain_step_tiles(const GemmChainArgs& a, int i) {
  int n = 0;
  for (int s = 0; s < a.n_stages; ++s) {
    const int r = i - a.st[s].lag;
    if (r >= 0 && r < a.n_blocks) n += a.st[s].n_tiles;
  }
  if (a.ln) {
    const int r = i - a.ln_lag;
    if (r >= 0 && r < a.n_blocks) n += 1;
  }
  return n;
}

// A position of the sequence as (step, index within the step), advanced in order. After every
// advance the cursor stands on a step that has tiles (steps without tiles are skipped), or on
// step n_steps once it is past the end; the walk never goes beyond n_steps.
struct ChainCursor {
  int step = 0, idx = 0;
  __device__ __forceinline__ void advance(const GemmChainArgs& a, int by) {
    idx += by;
    while (step < a.n_steps) {
      const int n = chain_step_tiles(a, step);
      if (idx < n) return;
      idx -= n;
      ++step;
    }
  }
};

struct ChainTile {
  int s;  // layer, or n_stages for a LayerNorm tile
  int r;  // row block
  int j;  // output column tile of the layer
};

__device__ __forceinline__ ChainTile chain_decode(const GemmChainArgs& a, const ChainCursor& c) {
  int idx = c.idx;
  for (int s = 0; s < a.n_stages; ++s) {
    const int r = c.step - a.st[s].lag;
    if (r >= 0 && r < a.n_blocks) {
      if (idx < a.st[s].n_tiles) return ChainTile{s, r, idx};
      idx -= a.st[s].n_tiles;
    }
  }
  return ChainTile{a.n_stages, c.step - a.ln_lag, 0};
}

// ------------------------------------------------------------------------ completion counters
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_gpu_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Wait until *p >= target (another tile has completed). Bounded like mbar_wait: on timeout the
// code goes to the status word, the CTA's abort flag is raised and false is returned.
__device__ __forceinline__ bool wait_counter(const int* p, int target, const WaitCtx& w, int code) {
  if (ld_acquire_gpu(p) >= target) return true;
  uint64_t t0 = 0;
  uint32_t spins = 0;
  while (true) {
    __nanosleep(128);
    if (ld_acquire_gpu(p) >= target) return true;
    if ((++spins & 15u) == 0) {
      if (*w.abort_flag) return false;
      const uint64_t now = globaltimer_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > w.timeout_ns) {
        atomicCAS(w.status, 0, code);
        *w.abort_flag = 1;
        return false;
      }
    }
  }
}

__device__ __forceinline__ void st_shared_cluster_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

// ------------------------------------------------------------------------------------------ kernel
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(320, 1)
    mlp_gemm_chain_kernel(const __grid_constant__ GemmChainMaps tm, const GemmChainArgs args) {
  using L = GemmChainLayout;
  constexpr int kS = L::kStages;
  constexpr int kT = L::kTidSlots;
  constexpr int kSignals = 2 * L::kEpiWarps;  // completion signals per tile: every epilogue warp of the pair
  // readers of each claimed position: the leader's MMA issuer, the peer's producer, every epilogue warp
  constexpr int kTidReaders = 2 + 2 * L::kEpiWarps;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* full = bars;            // [kS]
  uint64_t* empty = bars + 8;       // [kS]
  uint64_t* acc_full = bars + 16;   // [2]
  uint64_t* acc_empty = bars + 18;  // [2]
  uint64_t* mma_done = bars + 20;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 22);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 23);
  uint64_t* tid_full = bars + 24;   // [kT] a claimed position is in tid_val (this CTA's copy)
  uint64_t* tid_empty = bars + 28;  // [kT] (leader's) every reader has taken it
  volatile int* tid_val = reinterpret_cast<volatile int*>(bars + 32);   // [kT] claimed positions
  volatile int* tid_pack = reinterpret_cast<volatile int*>(bars + 34);  // [kT] their tiles, packed
  float* bias_s = reinterpret_cast<float*>(smem + L::kOffBias);
  float* head_s = reinterpret_cast<float*>(smem + L::kOffHead);  // [kMaxHead] weights, then the bias
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if ((smem_u32(smem) & 1023u) != 0) {
    pdl_wait_prior();
    if (threadIdx.x == 0) atomicCAS(args.status, 0, kDevBadSmemAlign);
    return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kS; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&acc_full[b]), 1);
      mbar_init(smem_u32(&acc_empty[b]), L::kEpiWarps * 2);
    }
    mbar_init(smem_u32(mma_done), 1);
    for (int i = 0; i < kT; ++i) {
      mbar_init(smem_u32(&tid_full[i]), 1);
      mbar_init(smem_u32(&tid_empty[i]), kTidReaders);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane < args.n_stages) {
    prefetch_tmap(&tm.a[lane]);
    prefetch_tmap(&tm.w[lane]);
    prefetch_tmap(&tm.out[lane]);
  }
  // everything above overlaps the previous kernel of the stream; global memory only from here
  pdl_wait_prior();
  if (threadIdx.x == 0) pdl_launch_dependents();
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_holder), 512);
    tmem_relinquish_pair();
  }
  for (int s = 0; s < args.n_stages; ++s) {
    const ChainStageArgs& st = args.st[s];
    for (int i = threadIdx.x; i < st.n; i += blockDim.x)
      bias_s[st.bias_off + i] = st.bias != nullptr ? load16(st.bias, i, st.bias_bf16) : 0.0f;
  }
  if (args.head_w != nullptr) {
    const int nl = args.st[args.n_stages - 1].n;
    for (int i = threadIdx.x; i < nl; i += blockDim.x) head_s[i] = load16(args.head_w, i, args.out_bf16);
    if (threadIdx.x == 0) head_s[L::kMaxHead] = args.head_b != nullptr ? load16(args.head_b, 0, args.out_bf16) : 0.0f;
  }
  tc_fence_before();
  cluster_sync_all();  // the peer's barriers are initialised before any remote arrival
  tc_fence_after();
  auto leader_bar = [&](const uint64_t* b) -> uint32_t { return mapa_shared(smem_u32(b), 0); };
  const uint32_t tmem_base = *tmem_holder;
  const WaitCtx wctx{args.status, abort_flag, args.timeout_ns};
  const int nb = args.n_blocks;
  auto counter = [&](int s, int r) { return args.counters + s * nb + r; };
  auto signal = [&](int* c, int v) {
    if (args.inject != 1) red_release_gpu_add(c, v);
  };
  // A claimed position and its tile: s | j << 3 | r << 8 (decoded once, by the claiming producer).
  struct Claim {
    int t;
    ChainTile tl;
  };
  auto unpack = [&](int t, int pk) -> Claim {
    return Claim{t, ChainTile{pk & 7, pk >> 8, (pk >> 3) & 31}};
  };
  // A reader's next claim (t >= total: the sequence is done; t < 0: the wait gave up). Called by
  // one thread per reader (lane 0 of the role), which then releases the slot.
  auto take = [&](int& slot, uint32_t& tph, int code) -> Claim {
    if (!mbar_wait<true>(smem_u32(&tid_full[slot]), tph, wctx, code)) return Claim{-1, ChainTile{0, -1, 0}};
    const Claim c = unpack(tid_val[slot], tid_pack[slot]);
    mbar_arrive_cluster(leader_bar(&tid_empty[slot]));
    if (++slot == kT) { slot = 0; tph ^= 1; }
    return c;
  };
  // read after write: all tiles of the previous layer for this row block have stored
  auto raw_target = [&](const ChainTile& tl) { return args.st[tl.s - 1].n_tiles * kSignals; };

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer (+ claims)
    // The leader claims positions (one ahead, so the claim's round trip overlaps the loads),
    // decodes them and publishes position and tile to both CTAs; the other CTA's producer reads
    // them. The next tile is fetched and its dependency tested a few stages before the current
    // tile's last load, so the next loads follow without a gap when the dependency is met.
    if (lane == 0) {
      const uint64_t keep = l2_policy_evict_last();
      int s = 0, slot = 0, prev = 0;
      uint32_t ph = 0, tph = 0;
      ChainCursor cur;
      int claimed = leader ? atomicAdd(args.next_tile, 1) : 0;
      auto fetch = [&]() -> Claim {
        if (!leader) return take(slot, tph, kDevTimeoutProducer);
        if (!mbar_wait<true>(smem_u32(&tid_empty[slot]), tph ^ 1, wctx, kDevTimeoutProducer))
          return Claim{-1, ChainTile{0, -1, 0}};
        Claim c{claimed, ChainTile{0, 0, 0}};
        if (c.t < args.total) {
          claimed = atomicAdd(args.next_tile, 1);
          cur.advance(args, c.t - prev);
          prev = c.t;
          c.tl = chain_decode(args, cur);
          if (c.tl.r < 0 || c.tl.r >= nb || cur.step >= args.n_steps) {
            atomicCAS(args.status, 0, kDevBadSchedule);
            *abort_flag = 1;
            c.t = -1;  // published as "gave up": every reader stops
          }
        }
        const int pk = c.tl.s | (c.tl.j << 3) | (c.tl.r << 8);
        tid_val[slot] = c.t;
        tid_pack[slot] = pk;
        st_shared_cluster_u32(mapa_shared(smem_u32(const_cast<int*>(&tid_val[slot])), 1), static_cast<uint32_t>(c.t));
        st_shared_cluster_u32(mapa_shared(smem_u32(const_cast<int*>(&tid_pack[slot])), 1), static_cast<uint32_t>(pk));
        mbar_arrive(smem_u32(&tid_full[slot]));
        mbar_arrive_cluster(mapa_shared(smem_u32(&tid_full[slot]), 1));
        if (++slot == kT) { slot = 0; tph ^= 1; }
        return c;
      };
      Claim cur_c = fetch();
      bool ready = false;  // cur_c's dependency was already seen complete
#pragma unroll 1
      while (cur_c.t >= 0 && cur_c.t < args.total) {
        const ChainTile tl = cur_c.tl;
        if (tl.s >= args.n_stages) {  // LayerNorm tile: no operands
          cur_c = fetch();
          ready = false;
          continue;
        }
        const ChainStageArgs& st = args.st[tl.s];
        int arow = tl.r * 256 + static_cast<int>(rank) * kBM;
        if (tl.s > 0) {
          if (!ready && !wait_counter(counter(tl.s - 1, tl.r), raw_target(tl), wctx, kDevTimeoutDependency)) break;
          fence_proxy_async_global();
          arow = (tl.r % args.st[tl.s - 1].ring_q) * 256 + static_cast<int>(rank) * kBM;
        }
        const int bblk = tl.j * (L::kBN / 64) + static_cast<int>(rank) * (L::kBN / 128);
        const int kpanels = (st.k + kPanel - 1) / kPanel;
        const int kp_fetch = kpanels > 3 ? kpanels - 3 : 0;
        Claim next{-1, ChainTile{0, -1, 0}};
        bool ok = true;
#pragma unroll 1
        for (int kp = 0; kp < kpanels; ++kp) {
          if (!mbar_wait<true>(smem_u32(&empty[s]), ph ^ 1, wctx, kDevTimeoutProducer)) { ok = false; break; }
          const uint32_t stg = smem_u32(smem + s * L::kStageBytes);
          if (leader) mbar_arrive_expect_tx(smem_u32(&full[s]), L::kStageBytes * 2);
          const uint32_t fb = leader_bar(&full[s]);
          tma_load_2d_pair(stg, &tm.a[tl.s], fb, kp * kPanel, arow, keep);
          tma_load_3d_pair(stg + L::kABytes, &tm.w[tl.s], fb, 0, kp * kPanel, bblk, keep);
          if (++s == kS) { s = 0; ph ^= 1; }
          if (kp == kp_fetch) {
            next = fetch();
            ready = false;
            if (next.t >= 0 && next.t < args.total && next.tl.s > 0 && next.tl.s < args.n_stages)
              ready = ld_acquire_gpu(counter(next.tl.s - 1, next.tl.r)) >= raw_target(next.tl);
          }
        }
        if (!ok) break;
        cur_c = next;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (pair leader)
    if (lane == 0 && leader) {
      int s = 0, g = 0, slot = 0;
      uint32_t ph = 0, tph = 0, eph[2] = {0, 0};
#pragma unroll 1
      while (true) {
        const Claim c = take(slot, tph, kDevTimeoutMma);
        if (c.t < 0 || c.t >= args.total) break;
        const ChainTile tl = c.tl;
        if (tl.s >= args.n_stages) continue;
        const ChainStageArgs& st = args.st[tl.s];
        const int b = g & 1;
        if (g >= 2) {
          if (!mbar_wait<true>(smem_u32(&acc_empty[b]), eph[b], wctx, kDevTimeoutMma)) break;
          eph[b] ^= 1;
        }
        ++g;
        tc_fence_after();
        const uint32_t idesc = make_idesc_f16(kBM * 2, L::kBN, st.a_bf16, 0, 1);
        const uint32_t d = tmem_base + b * L::kBN;
        const int kpanels = (st.k + kPanel - 1) / kPanel;
        bool ok = true;
#pragma unroll 1
        for (int kp = 0; kp < kpanels; ++kp) {
          if (!mbar_wait<true>(smem_u32(&full[s]), ph, wctx, kDevTimeoutMma)) { ok = false; break; }
          tc_fence_after();
          const uint32_t stg = smem_u32(smem + s * L::kStageBytes);
          const uint64_t adesc = make_sdesc_sw128(stg, 16, 1024);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t bdesc = make_sdesc_sw128(stg + L::kABytes + k * 2048, kPanel * 128, 1024);
            mma_ss_pair(d, adesc + static_cast<uint64_t>(k * 2), bdesc, idesc, (kp | k) != 0 ? 1u : 0u);
          }
          mma_commit_pair(smem_u32(&empty[s]), 0x3);
          if (++s == kS) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
        mma_commit_pair(smem_u32(&acc_full[b]), 0x3);
      }
      // drain: every issued MMA has completed before TMEM can be released
      mma_commit_pair(smem_u32(mma_done), 0x3);
    }
    if (lane == 0) {
      volatile int no_abort = 0;
      WaitCtx drain{args.status, &no_abort, args.timeout_ns};
      mbar_wait<true>(smem_u32(mma_done), 0, drain, kDevTimeoutMma);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue / LayerNorm tiles
    const int q = warp & 3;            // TMEM lane quarter
    const int eg = (warp - 2) >> 2;    // even / odd 32-column chunks
    const int ew = warp - 2;           // epilogue warp 0..7
    uint8_t* stg = smem + L::kOffStg + ew * L::kStgWarpBytes;
    int sb = 0, g = 0, slot = 0;
    uint32_t aph[2] = {0, 0}, tph = 0;
    // Completion of a tile's TMA stores is signalled one tile late (after the next tile's stores are
    // issued), so the warp does not sit out the store latency; a pending signal is flushed before
    // any wait that might depend on it.
    int pend_s = -1, pend_r = 0;
    auto flush = [&]() {
      if (pend_s < 0) return;
      if (lane == 0) {
        bulk_wait_group<0>();
        fence_proxy_async_global();
        signal(counter(pend_s, pend_r), 1);
      }
      __syncwarp();
      pend_s = -1;
    };
#pragma unroll 1
    while (true) {
      Claim c{0, ChainTile{0, 0, 0}};
      if (lane == 0) c = take(slot, tph, kDevTimeoutEpilogue);
      const int t = __shfl_sync(0xffffffffu, c.t, 0);
      if (t < 0 || t >= args.total) break;
      const ChainTile tl{__shfl_sync(0xffffffffu, c.tl.s, 0), __shfl_sync(0xffffffffu, c.tl.r, 0),
                         __shfl_sync(0xffffffffu, c.tl.j, 0)};
      if (tl.s >= args.n_stages) {
        // LayerNorm tile: this CTA's 128 rows of the row block, one warp per row
        const ChainStageArgs& lst = args.st[args.n_stages - 1];
        flush();
        // every lane reads the ring, so every lane acquires the counter
        const bool ready = wait_counter(counter(args.n_stages - 1, tl.r), lst.n_tiles * kSignals, wctx,
                                        kDevTimeoutDependency);
        if (!__all_sync(0xffffffffu, ready)) break;
        const float* ring = args.ln_ring + static_cast<size_t>((tl.r % lst.ring_q) * 256) * args.ln_n;
#pragma unroll 1
        for (int i = ew; i < kBM; i += L::kEpiWarps) {
          const int rb = static_cast<int>(rank) * kBM + i;
          const int64_t row = static_cast<int64_t>(tl.r) * 256 + rb;
          if (row >= args.m) break;
          layernorm_row_warp<1024>(ring + static_cast<size_t>(rb) * args.ln_n, args.gamma, args.beta, args.g_bf16,
                                   args.ln_eps, static_cast<uint16_t*>(args.out) + row * args.ln_n, args.out_bf16,
                                   lane);
        }
        __syncwarp();
        if (lane == 0) {
          __threadfence();
          signal(counter(args.n_stages, tl.r), 1);
        }
        continue;
      }
      const ChainStageArgs& st = args.st[tl.s];
      const int b = g & 1;
      ++g;
      // a tile that is not ready yet may wait on this warp's pending signal: flush it first (lane 0
      // decides, so the warp agrees)
      int ready_now = lane == 0 ? (mbar_test_wait_cluster(smem_u32(&acc_full[b]), aph[b]) ? 1 : 0) : 0;
      ready_now = __shfl_sync(0xffffffffu, ready_now, 0);
      if (!ready_now) flush();
      const bool got = mbar_wait<true>(smem_u32(&acc_full[b]), aph[b], wctx, kDevTimeoutEpilogue);
      if (!__all_sync(0xffffffffu, got)) break;
      aph[b] ^= 1;
      tc_fence_after();
      int okw = 1;
      if (st.ring_q > 0 && tl.r >= st.ring_q) {
        // write after read: the consumers of the row block that held this ring slot are done
        const int cs = tl.s + 1;
        const int need = (cs < args.n_stages ? args.st[cs].n_tiles : 1) * kSignals;
        flush();
        if (lane == 0) {
          okw = wait_counter(counter(cs, tl.r - st.ring_q), need, wctx, kDevTimeoutDependency) ? 1 : 0;
          fence_proxy_async_global();
        }
        if (__shfl_sync(0xffffffffu, okw, 0) == 0) break;
      }
      const int rl = static_cast<int>(rank) * kBM + q * 32;  // this warp's first row within the block
      const int64_t grow = static_cast<int64_t>(tl.r) * 256 + rl + lane;
      const int orow0 = st.ring_q > 0 ? (tl.r % st.ring_q) * 256 + rl : tl.r * 256 + rl;
      const bool store_ok = st.ring_q > 0 || orow0 < args.m;
      const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + b * L::kBN;
      // the sigmoid head needs whole rows: the even-chunk warp of each lane quarter reads all eight
      // chunks and the odd-chunk warp only releases the accumulator
      const bool head = st.out_kind == 2;
      const int c_first = head ? 0 : eg, c_step = head ? 1 : 2;
      const int c_end = (head && eg == 1) ? 0 : L::kBN / 32;
      if (head && eg == 1) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(leader_bar(&acc_empty[b]));
      }
      float hp = 0.0f;  // sigmoid head: this thread's dot product
      act_dispatch(st.act, [&](auto act_c) {
        constexpr int kAct = decltype(act_c)::value;
#pragma unroll 1
        for (int c = c_first; c < c_end; c += c_step) {
          uint32_t v[32];
          tmem_ld32(t_lane + c * 32, v);
          tmem_wait_ld();
          if (c + c_step >= L::kBN / 32) {  // this warp's part of the accumulator is read
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(leader_bar(&acc_empty[b]));
          }
          const int col0 = tl.j * L::kBN + c * 32;
          float y[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) y[i] = __uint_as_float(v[i]) + bias_s[st.bias_off + col0 + i];
          if (st.resid != nullptr && grow < args.m) {
            const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(st.resid) + grow * st.n + col0);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint4 w = __ldg(src + j);
              const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = unpack16x2(ws[e], st.resid_bf16);
                y[j * 8 + e * 2] += f.x;
                y[j * 8 + e * 2 + 1] += f.y;
              }
            }
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) y[i] = act_t<kAct>(y[i]);
          if (st.out_kind == 2) {
#pragma unroll
            for (int i = 0; i < 32; ++i) hp = fmaf(y[i], head_s[col0 + i], hp);
          } else if (st.out_kind == 1) {
            // 32 x 32 fp32 tile, 128-byte rows in the SWIZZLE_128B layout of the output map
            if (lane == 0) bulk_wait_group_read<0>();
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 8; ++j)
              *reinterpret_cast<float4*>(stg + lane * 128 + ((j ^ (lane & 7)) * 16)) =
                  make_float4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              if (store_ok) tma_store_2d(&tm.out[tl.s], smem_u32(stg), col0, orow0);
              bulk_commit_group();
            }
          } else {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              pk[i] = st.out_bf16 ? Elem<__nv_bfloat16>::pack(y[2 * i], y[2 * i + 1])
                                  : Elem<__half>::pack(y[2 * i], y[2 * i + 1]);
            uint8_t* sbuf = stg + sb * 2048;
            if (lane == 0) bulk_wait_group_read<1>();  // the store that last read buffer sb is done
            __syncwarp();
            stage_chunk32(sbuf, lane, pk);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              if (store_ok) tma_store_2d(&tm.out[tl.s], smem_u32(sbuf), col0, orow0);
              bulk_commit_group();
            }
            sb ^= 1;
          }
        }
      });
      if (head && eg == 0 && grow < args.m) {
        const float o = act_t<kActSigmoid>(hp + head_s[L::kMaxHead]);
        uint16_t* dst = static_cast<uint16_t*>(args.out) + grow;
        if (args.out_bf16) {
          const __nv_bfloat16 h = __float2bfloat16_rn(o);
          *dst = *reinterpret_cast<const uint16_t*>(&h);
        } else {
          const __half h = __float2half_rn(o);
          *dst = *reinterpret_cast<const uint16_t*>(&h);
        }
      }
      if (head) {
        // plain stores by the lanes: fenced and signalled now (one tile in eleven)
        flush();
        __threadfence();
        __syncwarp();
        if (lane == 0) signal(counter(tl.s, tl.r), 1);
      } else {
        // the previous tile's stores are the groups before this tile's four
        if (pend_s >= 0) {
          if (lane == 0) {
            bulk_wait_group<L::kBN / 64>();
            fence_proxy_async_global();
            signal(counter(pend_s, pend_r), 1);
          }
          __syncwarp();
        }
        pend_s = tl.s;
        pend_r = tl.r;
      }
    }
    flush();
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }
  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while the pair's MMAs may still read its memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 512);
  }
}

}  // namespace gp
