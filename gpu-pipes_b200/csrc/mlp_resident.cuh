// Fused MLP chain with weights resident in shared memory ("narrow" chains: hidden width <= 128).
//
// Covers the reference apps whose every layer is at most 128 wide:
//   mgn_fullmlp  apps/mgn_fullmlp/pipelined/mgn_fullmlp_pl.cuh:205-252   384->128->128->128 + LN
//   mgn_linears  apps/mgn_linears/pipelined/mgn_linears_pl.cuh:176-212   384->128->128->128
//   test_mlp     apps/test_mlp/pipelined/test_mlp_pl.cuh:127-161         128->128->128->128
// and the MeshGraphNet node MLP (256->128->128->128 + LN).
//
// Where the reference pins each layer to its own CTA and passes 128x128 activation tiles between
// CTAs through L2-resident ring queues (common/mpmcq.cuh, common/pipes.cuh), this kernel runs the
// whole chain for a 128-row tile inside one persistent CTA:
//
//   warp 0      TMA producer: all weights once (smem-resident for the CTA's lifetime), then the
//               x tiles as 128x64 K panels through an mbarrier ring.
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer.
//   warps 2-9   two epilogue groups of four warps (one per TMEM accumulator buffer); thread t of a
//               group owns row t of its tile (TMEM lane t).
//
// Two row tiles are in flight (TMEM buffers b = 0, 1), so the tensor core works on one tile while
// the epilogue of the other runs. Per buffer (256 TMEM columns):
//   cols [0, N)          fp32 accumulator of the current layer
//   cols [128, 128+N/2)  16-bit activation of the previous layer, two values per column; it is the
//                        A operand (tcgen05.mma A-from-TMEM) of the next layer.
// Hidden activations therefore never leave the SM: HBM traffic is x, the weights once per CTA,
// and the final output.
//
// Layer 0 is A[smem x panel, K-major SW128] x B[smem W, N-major SW128]; layers >= 1 are
// A[TMEM activation] x B[smem W]. The epilogue of the last layer applies bias, activation or
// LayerNorm (thread-local: one thread holds one full row) and stores through a per-warp swizzled
// staging buffer with TMA.
#pragma once

#include "chain_common.cuh"
#include "gp_ptx.cuh"

namespace gp {

template <int K0_, int N_, int NL_>
struct ResidentLayout {
  static constexpr int K0 = K0_, N = N_, NL = NL_;
  static_assert(K0 % kPanel == 0 && K0 >= kPanel, "K0 must be a multiple of 64");
  static_assert(N % kPanel == 0 && N >= 64 && N <= 128, "hidden width must be 64 or 128");
  static_assert(NL >= 1 && NL <= kMaxLayers, "layer count");
  static constexpr int kW0Bytes = K0 * N * 2;
  static constexpr int kWhBytes = N * N * 2;
  static constexpr int kWBytes = kW0Bytes + (NL - 1) * kWhBytes;
  static constexpr int kStageBytes = 32 * 128;  // per epilogue warp: 32 rows x 64 cols x 2 B
  static constexpr int kNumEpiWarps = 8;
  static constexpr int kStgBytes = kNumEpiWarps * kStageBytes;
  static constexpr int kBarBytes = 256;
  static constexpr int kAlignSlack = 1024;
  static constexpr int kXStagesRaw =
      (kSmemLimit - kAlignSlack - kBarBytes - kWBytes - kStgBytes) / kPanelBytes;
  static constexpr int kXStages = kXStagesRaw > 8 ? 8 : kXStagesRaw;
  static_assert(kXStages >= 2, "weights do not fit in shared memory");
  // offsets from the 1024-aligned base
  static constexpr int kOffW = 0;
  static constexpr int kOffX = kOffW + kWBytes;
  static constexpr int kOffStg = kOffX + kXStages * kPanelBytes;
  static constexpr int kOffBar = kOffStg + kStgBytes;
  static constexpr int kSmemBytes = kOffBar + kBarBytes + kAlignSlack;
  static_assert(kSmemBytes <= kSmemLimit, "shared memory budget");
  static constexpr int kThreads = 320;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr int kBufCols = 256;
  static constexpr int kActCol = 128;
};

__device__ __forceinline__ uint32_t w_layer_offset(int l, int w0_bytes, int wh_bytes) {
  return l == 0 ? 0u : static_cast<uint32_t>(w0_bytes + (l - 1) * wh_bytes);
}

// ------------------------------------------------------------------------------------------------
// Epilogue pieces. `v` holds one row's fp32 accumulators (thread = row), 32 columns per block.
// ------------------------------------------------------------------------------------------------
template <int ACT>
__device__ __forceinline__ float act_c(float v) {
  return apply_act(ACT, v);
}

template <typename T>
__device__ __forceinline__ void unpack2(uint32_t bits, float& lo, float& hi) {
  lo = Elem<T>::to_f(*reinterpret_cast<const T*>(&bits));
  hi = Elem<T>::to_f(*(reinterpret_cast<const T*>(&bits) + 1));
}

// bias + activation, packed to 16 bits and written to TMEM (two values per column).
template <typename T, int N, int ACT>
__device__ __forceinline__ void epi_hidden(const uint32_t (&v)[N / 32][32], const uint32_t* bias2,
                                           uint32_t t_act) {
#pragma unroll
  for (int c = 0; c < N / 32; ++c) {
    uint32_t pk[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float b0 = 0.f, b1 = 0.f;
      if (bias2 != nullptr) unpack2<T>(__ldg(bias2 + c * 16 + j), b0, b1);
      pk[j] = Elem<T>::pack(act_c<ACT>(__uint_as_float(v[c][2 * j]) + b0),
                            act_c<ACT>(__uint_as_float(v[c][2 * j + 1]) + b1));
    }
    tmem_st16(t_act + c * 16, pk);
  }
}

template <typename T, int N>
__device__ __forceinline__ void epi_bias(const uint32_t (&v)[N / 32][32], const uint32_t* bias2,
                                         float (&y)[N]) {
#pragma unroll
  for (int c = 0; c < N / 32; ++c)
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float b0 = 0.f, b1 = 0.f;
      if (bias2 != nullptr) unpack2<T>(__ldg(bias2 + c * 16 + j), b0, b1);
      y[c * 32 + 2 * j] = __uint_as_float(v[c][2 * j]) + b0;
      y[c * 32 + 2 * j + 1] = __uint_as_float(v[c][2 * j + 1]) + b1;
    }
}

template <int N, int ACT>
__device__ __forceinline__ void apply_act_row(float (&y)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) y[i] = act_c<ACT>(y[i]);
}

// LayerNorm of one row held entirely by this thread: biased variance, two passes
// (mean, then squared deviations), as torch.nn.LayerNorm and common/layer_norm_v2.cuh:34-68.
template <typename T, int N>
__device__ __forceinline__ void row_layernorm(float (&y)[N], const void* gamma, const void* beta,
                                              float eps) {
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i) sum += y[i];
  const float mean = sum * (1.0f / N);
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const float d = y[i] - mean;
    sq += d * d;
  }
  const float rstd = rsqrtf(sq * (1.0f / N) + eps);
  const uint32_t* g2 = reinterpret_cast<const uint32_t*>(gamma);
  const uint32_t* be2 = reinterpret_cast<const uint32_t*>(beta);
#pragma unroll
  for (int i = 0; i < N / 2; ++i) {
    float g0 = 1.f, g1 = 1.f, e0 = 0.f, e1 = 0.f;
    if (g2 != nullptr) unpack2<T>(__ldg(g2 + i), g0, g1);
    if (be2 != nullptr) unpack2<T>(__ldg(be2 + i), e0, e1);
    y[2 * i] = (y[2 * i] - mean) * rstd * g0 + e0;
    y[2 * i + 1] = (y[2 * i + 1] - mean) * rstd * g1 + e1;
  }
}

// Write 64 values of this thread's row into a 32-row x 128-byte staging tile with the TMA
// SWIZZLE_128B pattern (16-byte chunk j of row r lands at chunk j ^ (r % 8)).
template <typename T>
__device__ __forceinline__ void stage_row_chunk64(uint8_t* stg, int lane, const float* y) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint4 pk;
    pk.x = Elem<T>::pack(y[j * 8 + 0], y[j * 8 + 1]);
    pk.y = Elem<T>::pack(y[j * 8 + 2], y[j * 8 + 3]);
    pk.z = Elem<T>::pack(y[j * 8 + 4], y[j * 8 + 5]);
    pk.w = Elem<T>::pack(y[j * 8 + 6], y[j * 8 + 7]);
    *reinterpret_cast<uint4*>(stg + lane * 128 + ((j ^ (lane & 7)) * 16)) = pk;
  }
}

template <typename T, int K0, int N, int NL, uint32_t ACTS, int TAIL>
__global__ void __launch_bounds__(320, 1)
    mlp_resident_kernel(const __grid_constant__ TensorMaps tm, const ChainArgs args) {
  using L = ResidentLayout<K0, N, NL>;
  constexpr int kXS = L::kXStages;
  constexpr int kPanels0 = K0 / kPanel;
  constexpr uint32_t kIdesc = make_idesc_f16(kBM, N, Elem<T>::kIsBf16, 0, 1);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  // barrier slots
  uint64_t* x_full = bars;                // [kXS]
  uint64_t* x_empty = bars + 8;           // [kXS]
  uint64_t* w_full = bars + 16;           // [1]
  uint64_t* acc_full = bars + 17;         // [2]
  uint64_t* act_ready = bars + 19;        // [2]
  uint64_t* mma_done = bars + 21;         // [1]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 24);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 25);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kXS; ++s) {
      mbar_init(smem_u32(&x_full[s]), 1);
      mbar_init(smem_u32(&x_empty[s]), 1);
    }
    mbar_init(smem_u32(w_full), 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&acc_full[b]), 1);
      mbar_init(smem_u32(&act_ready[b]), 4);
    }
    mbar_init(smem_u32(mma_done), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm.x);
    prefetch_tmap(&tm.out);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_holder), L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  const WaitCtx wctx{args.status, abort_flag, args.timeout_ns};
  const int num_tiles = args.num_tiles;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      const uint64_t keep = l2_policy_evict_last();
      const uint64_t stream = l2_policy_evict_first();
      mbar_arrive_expect_tx(smem_u32(w_full), L::kWBytes);
#pragma unroll 1
      for (int l = 0; l < NL; ++l) {
        const int kl = l == 0 ? K0 : N;
        const uint32_t wbase = smem_u32(smem + L::kOffW + w_layer_offset(l, L::kW0Bytes, L::kWhBytes));
        for (int kp = 0; kp < kl / kPanel; ++kp)
          for (int nb = 0; nb < N / kPanel; ++nb)
            tma_load_2d_hint(wbase + nb * (kl * 128) + kp * (kPanel * 128), &tm.w[l],
                             smem_u32(w_full), nb * kPanel, kp * kPanel, keep);
      }
      int s = 0;
      uint32_t ph = 0;
#pragma unroll 1
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
#pragma unroll 1
        for (int p = 0; p < kPanels0; ++p) {
          if (!mbar_wait(smem_u32(&x_empty[s]), ph ^ 1, wctx, kDevTimeoutProducer)) goto producer_done;
          if (!args.inject) {
            mbar_arrive_expect_tx(smem_u32(&x_full[s]), kPanelBytes);
            tma_load_2d_hint(smem_u32(smem + L::kOffX + s * kPanelBytes), &tm.x,
                             smem_u32(&x_full[s]), p * kPanel, tile * kBM, stream);
          }
          if (++s == kXS) { s = 0; ph ^= 1; }
        }
      }
    producer_done:;
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(smem_u32(w_full), 0, wctx, kDevTimeoutWeights);
      tc_fence_after();
      const uint32_t wsm = smem_u32(smem + L::kOffW);
      const uint32_t xsm = smem_u32(smem + L::kOffX);
      int s = 0;
      uint32_t ph = 0;
      uint32_t ready_ph[2] = {0, 0};
      bool first[2] = {true, true};
#pragma unroll 1
      for (int pair = blockIdx.x; ok && pair < num_tiles; pair += 2 * gridDim.x) {
#pragma unroll 1
        for (int l = 0; ok && l < NL; ++l) {
#pragma unroll 1
          for (int b = 0; ok && b < 2; ++b) {
            const int tile = pair + b * gridDim.x;
            if (tile >= num_tiles) continue;
            if (!first[b]) {
              if (!mbar_wait(smem_u32(&act_ready[b]), ready_ph[b], wctx, kDevTimeoutMma)) { ok = false; break; }
              ready_ph[b] ^= 1;
            }
            first[b] = false;
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + b * L::kBufCols;
            if (l == 0) {
              for (int p = 0; p < kPanels0; ++p) {
                if (!mbar_wait(smem_u32(&x_full[s]), ph, wctx, kDevTimeoutMma)) { ok = false; break; }
                tc_fence_after();
                const uint64_t adesc = make_sdesc_sw128(xsm + s * kPanelBytes, 16, 1024);
#pragma unroll
                for (int k = 0; k < kPanel / 16; ++k) {
                  const int kk = p * (kPanel / 16) + k;  // 16-row K step within W0
                  const uint64_t bdesc = make_sdesc_sw128(wsm + kk * 2048, K0 * 128, 1024);
                  mma_ss(d_tmem, adesc + static_cast<uint64_t>(k * 2), bdesc, kIdesc,
                         (p | k) != 0 ? 1u : 0u);
                }
                mma_commit(smem_u32(&x_empty[s]));
                if (++s == kXS) { s = 0; ph ^= 1; }
              }
              if (!ok) break;
            } else {
              const uint32_t wl = wsm + w_layer_offset(l, L::kW0Bytes, L::kWhBytes);
              const uint32_t a_tmem = tmem_base + b * L::kBufCols + L::kActCol;
#pragma unroll
              for (int k = 0; k < N / 16; ++k) {
                const uint64_t bdesc = make_sdesc_sw128(wl + k * 2048, N * 128, 1024);
                mma_ts(d_tmem, a_tmem + k * 8, bdesc, kIdesc, k != 0 ? 1u : 0u);
              }
            }
            mma_commit(smem_u32(&acc_full[b]));
          }
        }
      }
      // drain: every issued MMA has completed before TMEM can be released
      mma_commit(smem_u32(mma_done));
      WaitCtx drain{args.status, abort_flag, args.timeout_ns};
      volatile int zero = 0;
      drain.abort_flag = &zero;  // drain even after an abort
      mbar_wait(smem_u32(mma_done), 0, drain, kDevTimeoutMma);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..9)
    const int g = (warp - 2) >> 2;         // TMEM buffer served by this group
    const int q = warp & 3;                // TMEM lane quarter accessible to this warp
    uint8_t* stg = smem + L::kOffStg + (warp - 2) * L::kStageBytes;
    const uint32_t stg_u32 = smem_u32(stg);
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + g * L::kBufCols;
    uint32_t acc_ph = 0;
    bool ok = true;
#pragma unroll 1
    for (int tile = blockIdx.x + g * gridDim.x; ok && tile < num_tiles; tile += 2 * gridDim.x) {
#pragma unroll 1
      for (int l = 0; l < NL; ++l) {
        if (!mbar_wait(smem_u32(&acc_full[g]), acc_ph, wctx, kDevTimeoutEpilogue)) { ok = false; break; }
        acc_ph ^= 1;
        tc_fence_after();
        uint32_t v[N / 32][32];
#pragma unroll
        for (int c = 0; c < N / 32; ++c) tmem_ld32(t_lane + c * 32, v[c]);
        tmem_wait_ld();
        const uint32_t* bias2 = reinterpret_cast<const uint32_t*>(args.bias[l]);
        const int act = static_cast<int>((ACTS >> (4 * l)) & 15u);
        if (l + 1 < NL) {
          // hidden layer: bias + activation -> 16-bit activation in TMEM (next layer's A)
          switch (act) {
            case kActRelu: epi_hidden<T, N, kActRelu>(v, bias2, t_lane + L::kActCol); break;
            case kActGeluTanh: epi_hidden<T, N, kActGeluTanh>(v, bias2, t_lane + L::kActCol); break;
            case kActSilu: epi_hidden<T, N, kActSilu>(v, bias2, t_lane + L::kActCol); break;
            case kActSigmoid: epi_hidden<T, N, kActSigmoid>(v, bias2, t_lane + L::kActCol); break;
            default: epi_hidden<T, N, kActNone>(v, bias2, t_lane + L::kActCol); break;
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&act_ready[g]));
        } else {
          // last layer: the accumulator is in registers; release the TMEM buffer first
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&act_ready[g]));
          float y[N];
          epi_bias<T, N>(v, bias2, y);
          if constexpr (TAIL == kTailLayerNorm) {
            row_layernorm<T, N>(y, args.gamma, args.beta, args.ln_eps);
          } else {
            switch (act) {
              case kActRelu: apply_act_row<N, kActRelu>(y); break;
              case kActGeluTanh: apply_act_row<N, kActGeluTanh>(y); break;
              case kActSilu: apply_act_row<N, kActSilu>(y); break;
              case kActSigmoid: apply_act_row<N, kActSigmoid>(y); break;
              default: break;
            }
          }
          // store: per 64-column chunk, swizzled staging (SW128) then a 32x64 TMA store
          const int row0 = tile * kBM + q * 32;
#pragma unroll
          for (int h = 0; h < N / 64; ++h) {
            if (lane == 0) bulk_wait_group_read<0>();
            __syncwarp();
            stage_row_chunk64<T>(stg, lane, y + h * 64);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0 && row0 < args.m) {
              tma_store_2d(&tm.out, stg_u32, h * 64, row0);
              bulk_commit_group();
            }
          }
        }
      }
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

}  // namespace gp
