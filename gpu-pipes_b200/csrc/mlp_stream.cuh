// Fused MLP chain with weights streamed from L2 ("wide" chains: hidden layers up to 512 wide).
//
// Covers the reference apps whose weights do not fit in one SM's shared memory:
//   dlrm_botmlp  apps/dlrm_botmlp/pipelined/dlrm_botmlp_pl.cuh:139-173  13(16)->512->256->128, ReLU
//   gc_edges     apps/gc_edges/pipelined/gc_edges_pl.cuh:112-142        1536->512->512 + LN(512)
//   gc_nodes     (same kernel family, K0 = 1024)
//   nerf_a       apps/nerf_a/pipelined/nerf_a_pl.cuh:183-227            64->256 x5, [h || x] -> 256,
//                                                                       256 x2, then a 256->4 head
// The reference gives every layer (and the concat / LN) its own CTA and moves activation tiles
// between them through L2 ring queues; the concat is a separate copy stage
// (common/pipe_concat.cuh:47-74). Here one persistent CTA runs the whole chain for a 128-row tile:
//
//   warp 0      TMA producer: x tiles (a resident 64-column tile, or a ring of 64-column panels
//               for wide inputs) and every layer's weights as 32-row x (<=256)-column stages
//               through an mbarrier ring (L2-resident: every CTA streams the same weights).
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer.
//   warps 2-9   epilogue, two warps per TMEM lane quarter: thread t of a quarter's pair owns row
//               t of the tile (TMEM lane t); warp group 0 drains the even 32-column accumulator
//               chunks, group 1 the odd ones, so two warps per scheduler hide each other's
//               TMEM-load and math latency. Row sums for the LayerNorm and the head's partial
//               dot products are combined through shared memory.
//
// Activations never leave the SM: the epilogue of layer l writes bias + activation of the fp32
// accumulator as 16-bit values straight into shared memory, in the K-major SWIZZLE_128B layout
// the next layer's MMA reads as its A operand. The skip concat of NeRF is free: the A operand of
// that layer is the activation panels followed by the resident x panel. Accumulators hold up to
// 512 fp32 columns (N = 512 runs as two 256-wide MMAs per K step). Tails: LayerNorm in two passes
// over TMEM (row statistics, then normalise), or a narrow head (N < 64, e.g. NeRF 256 -> 4,
// DLRM 256 -> 1) computed on CUDA cores from the last hidden row held by the thread.
#pragma once

#include "chain_common.cuh"
#include "gp_ptx.cuh"
#include "mlp_resident.cuh"

namespace gp {

constexpr int kTailHead = 3;  // narrow output layer on CUDA cores (stream kernel only)

// Chain description used as a template argument (HALVES: 2 = each layer's output is computed
// and drained as two column halves so the epilogue of one overlaps the MMAs of the other;
// 1 = one pass per layer):
//   using T;  NL (tensor-core layers); K(l), N(l), ACT(l); SKIP (layer whose A operand is
//   [act || x], 0 = none); TAIL (kTailNone / kTailLayerNorm / kTailResidualLN / kTailHead; the
//   residual rows [M, N_last] of kTailResidualLN come from args.resid); HEAD_N, HEAD_ACT;
//   HIDDEN_F16: with bf16 data, keep hidden activations in fp16 (11-bit mantissa instead of 8)
//   and run layers >= 1 as fp16 x fp16 MMAs on fp16 copies of their weights (bf16 -> fp16 is
//   exact for weights within fp16 range). Input, first layer and output stay bf16.
//   OUT_N (optional): stored output columns, a multiple of 32 not above N_last (default N_last);
//   the columns beyond it are computed and dropped, the output rows are OUT_N wide.
template <class C, class = void>
struct OutCols {
  static constexpr int value = C::N(C::NL - 1);
};
template <class C>
struct OutCols<C, std::void_t<decltype(C::OUT_N)>> {
  static constexpr int value = C::OUT_N;
};

//   EPI_PAIRS (optional, default true): hidden-layer epilogues load two of a warp's 32-column
//   chunks behind one TMEM wait (GraphCast 3.79 -> 3.65 ms, NeRF 4.73 -> 4.66 ms; DLRM bottom
//   0.233 -> 0.242 ms, so that chain sets it false).
template <class C, class = void>
struct EpiPairs {
  static constexpr bool value = true;
};
template <class C>
struct EpiPairs<C, std::void_t<decltype(C::EPI_PAIRS)>> {
  static constexpr bool value = C::EPI_PAIRS;
};

//   SIDE (optional, default -1): a hidden layer whose output (bias + activation) is a second
//   result, stored straight from registers to args.out2 ([M, N(SIDE)] rows) instead of the
//   activation buffer; the layer after it reads the same activation as SIDE did (a branch off the
//   chain, e.g. NeRF's alpha head off the trunk). Needs SPLIT_ACT.
template <class C, class = void>
struct SideLayer {
  static constexpr int value = -1;
};
template <class C>
struct SideLayer<C, std::void_t<decltype(C::SIDE)>> {
  static constexpr int value = C::SIDE;
};

//   SKIP2 (optional, default 0): a layer whose last 64-column A panel is the second input
//   (args x2 through tm.x2, [M, <= 64] rows, zero filled to 64 columns), e.g. NeRF's view
//   directions concatenated to the bottleneck. The panel is loaded into the resident x buffer
//   once x's last reader (layer 0 or SKIP) is done, so it costs no shared memory.
template <class C, class = void>
struct Skip2Layer {
  static constexpr int value = 0;
};
template <class C>
struct Skip2Layer<C, std::void_t<decltype(C::SKIP2)>> {
  static constexpr int value = C::SKIP2;
};

//   WROWS(l) (optional, default K(l)): rows of weight l present in memory; the rows from WROWS(l)
//   to K(l) are read as zeros (the TMA box reaches past the tensor), which pads a K that is not a
//   whole number of 16-row steps without a copy.
template <class C, class = void>
struct WeightRows {
  static constexpr int get(int l) { return C::K(l); }
};
template <class C>
struct WeightRows<C, std::void_t<decltype(C::WROWS(0))>> {
  static constexpr int get(int l) { return C::WROWS(l); }
};

template <class C, int CG = 1>
struct StreamLayout {
  static constexpr int NL = C::NL;
  static constexpr int K0 = C::K(0);
  static constexpr bool kXRes = K0 <= kPanel;  // whole x tile resident (one 64-column panel)
  static constexpr int kOutN = OutCols<C>::value;
  static_assert(kOutN % 32 == 0 && kOutN <= C::N(C::NL - 1), "OUT_N");
  __host__ __device__ static constexpr int maxN() {
    int m = 0;
    for (int l = 0; l < NL; ++l) m = C::N(l) > m ? C::N(l) : m;
    return m;
  }
  __host__ __device__ static constexpr int actW() {  // widest activation that feeds a later layer
    int m = 64;
    for (int l = 0; l + 1 < NL; ++l) m = C::N(l) > m ? C::N(l) : m;
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
  static constexpr int kMaxN = maxN();
  static_assert(kMaxN <= 512, "accumulators are at most 512 columns");
  static constexpr int NH = C::HALVES;  // output halves per layer (1 or 2)
  static_assert(NH == 1 || NH == 2, "one or two output halves");
  static constexpr int kNB = kMaxN / NH;  // N columns per MMA / per B stage (one output half)
  static_assert(kNB <= 256, "an output half is at most 256 columns");
  __host__ __device__ static constexpr bool halvesOk() {
    for (int l = 0; l < NL; ++l)
      if (C::N(l) % (64 * C::HALVES) != 0) return false;
    return true;
  }
  static_assert(halvesOk(), "every layer width must split into two halves of whole 64-column panels");
  // SPLIT_ACT (one pass per layer, N <= 256): accumulators alternate between TMEM columns
  // [0, 256) and [256, 512) from layer to layer, and each epilogue releases the activation panels
  // in two halves, so the next layer's MMAs start on the first half of its K while the epilogue
  // still writes the second.
  static constexpr bool kSplit = C::SPLIT_ACT;
  static_assert(!kSplit || (NH == 1 && maxN() <= 256), "SPLIT_ACT: one pass per layer, N <= 256");
  static constexpr int kActBytes = kBM * actW() * 2;
  // resident x: one buffer. x is released once its last reader (layer 0, or the skip layer) has
  // run, so the next tile's x loads while the remaining layers run; the 16 KB saved go to the
  // weight ring.
  static constexpr int kXBytes = kXRes ? kPanelBytes : 0;
  __host__ __device__ static constexpr bool pairOk() {
    for (int l = 0; l < NL; ++l)
      if ((C::N(l) / NH) % 128 != 0) return false;
    return true;
  }
  static_assert(CG == 1 || (CG == 2 && pairOk()), "CTA pairs need output halves of 128-column multiples");
  static constexpr int kBiasBytes = ((biasFloats() * 4 + 1023) / 1024) * 1024;
  static constexpr bool kLN = C::TAIL == kTailLayerNorm || C::TAIL == kTailResidualLN;
  static constexpr int kLnBytes = kLN ? 2 * C::N(NL - 1) * 4 : 0;
  static constexpr int kHeadPad = ((C::HEAD_N + 3) / 4) * 4;  // head outputs, padded to float4
  static constexpr int kHeadBytes = C::TAIL == kTailHead ? (C::N(NL - 1) * kHeadPad * 4 + 64 * 4) : 0;
  static constexpr int kEpiWarps = 8;
  static constexpr int kStageBytes = 32 * 64;  // per epilogue warp output staging (32 x 32 x 2 B)
  // Output staging inside the activation buffer, two 2 KB buffers per warp in its own lane
  // quarter of two consecutive panels from kStgPanel0: for LayerNorm tails panels 0 and 1 (all of
  // the last layer's MMAs are complete before its epilogue stages anything); otherwise the first
  // panels the last layer does not read (its A operand is panels 0 .. K/64 - 1).
  static constexpr int kStgPanel0 = kLN ? 0 : (C::K(NL - 1) + kPanel - 1) / kPanel;
  static constexpr bool kStgInAct = C::TAIL != kTailHead && (C::SKIP == 0 || C::SKIP != NL - 1) &&
                                    actW() >= (kStgPanel0 + 2) * kPanel;
  static constexpr int kStgBytes = (C::TAIL == kTailHead || kStgInAct) ? 0 : kEpiWarps * kStageBytes;
  // cross-group exchange: LayerNorm (sum, sum of squares) or head partial sums, per row
  static constexpr int kXchgBytes =
      C::TAIL == kTailHead ? kBM * kHeadPad * 4 : (kLN ? 2 * kBM * 8 : 0);
  static constexpr int kBarBytes = 256;  // 32 eight-byte slots (see the kernel)
  static constexpr int kFixed = kActBytes + kXBytes + kBiasBytes + kLnBytes + kHeadBytes +
                                kXchgBytes + kStgBytes + kBarBytes + 1024;  // + alignment of the staging area
  // ring of x panels (streamed x only), then as many B stages as fit (at most 8). A stage holds
  // kBK weight rows of one output half (a CTA pair runs 256-row MMAs and each CTA stages half of
  // the columns) and arrives as ONE 3-D TMA request: TMA cost is largely per request, so 64-row
  // stages are used whenever three of them fit, 32-row stages otherwise.
  static constexpr int kXStages = kXRes ? 0 : 2;
  static constexpr int kXSlots = kXRes ? 1 : kXStages;  // x buffers cycled by xs
  static constexpr int kSide = SideLayer<C>::value;
  static constexpr int kSkip2 = Skip2Layer<C>::value;
  static constexpr int kLastXLayer = C::SKIP != 0 ? C::SKIP : 0;  // x's last reader
  // the second input is loaded two layers ahead of its reader (never before x's last reader)
  static constexpr int kLoadX2Layer = kSkip2 - 2 > kLastXLayer + 1 ? kSkip2 - 2 : kLastXLayer + 1;
  static_assert(kSide < 0 || (kSplit && kSide > 0 && kSide + 1 < NL), "SIDE: a hidden layer of a SPLIT_ACT chain");
  static_assert(kSkip2 == 0 || (kXRes && CG == 1 && kSkip2 > kLastXLayer + 1 && kSkip2 < NL),
                "SKIP2: a resident-x chain, after x's last reader");
  static constexpr int kRingBytes = kSmemLimit - kFixed - kXStages * kPanelBytes;
  // Stage rows: 128 (two K panels per request; only where x is resident, since a streamed x
  // panel is consumed with its own weight rows), else 64, else 32 -- the largest of which two
  // stages fit. The weight ring delivers about one stage per fixed interval whatever its size or
  // the ring depth, so larger stages carry more bytes per interval (DLRM bottom: 0.269 ms with
  // four 32-row stages, 0.235 with two 64-row ones).
  static constexpr int kBK = (kXRes && kRingBytes / (128 * kNB * 2 / CG) >= 2) ? 128
                             : kRingBytes / (64 * kNB * 2 / CG) >= 2 ? 64 : 32;
  static constexpr int kSub = kBK >= kPanel ? 1 : kPanel / kBK;  // stages per K panel (kBK <= 64)
  static_assert(C::SKIP == 0 || kXRes, "skip concat reads a resident x panel");
  static constexpr int kBStageBytes = kBK * kNB * 2 / CG;
  static constexpr int kBStagesRaw = (kSmemLimit - kFixed - kXStages * kPanelBytes) / kBStageBytes;
  static constexpr int kBStages = kBStagesRaw > 8 ? 8 : kBStagesRaw;
  static_assert(kBStages >= 2, "shared memory budget");
  static constexpr int kOffAct = 0;
  static constexpr int kOffX = kOffAct + kActBytes;                     // resident x or x ring
  static constexpr int kOffB = kOffX + (kXRes ? kXBytes : kXStages * kPanelBytes);
  static constexpr int kOffBias = kOffB + kBStages * kBStageBytes;
  static constexpr int kOffLn = kOffBias + kBiasBytes;
  static constexpr int kOffHead = kOffLn + kLnBytes;
  static constexpr int kOffXchg = kOffHead + kHeadBytes;
  static constexpr int kOffStg = ((kOffXchg + kXchgBytes + 1023) / 1024) * 1024;
  static constexpr int kOffBar = ((kOffStg + kStgBytes + 15) / 16) * 16;
  static constexpr int kSmemBytes = kOffBar + kBarBytes;
  static_assert(kSmemBytes <= kSmemLimit, "shared memory budget");
  static_assert(kOffX % 1024 == 0 && kOffB % 1024 == 0 && kOffStg % 512 == 0, "alignment");
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static_assert(kThreads == 320, "launch bounds of mlp_stream_kernel");
};

// Number of 16-wide K steps of layer l in 64-column panel p, and in its BK-row part h.
template <class C, int BK>
__host__ __device__ constexpr int ksteps_in(int l, int p, int h) {
  const int total = C::K(l) / 16;
  int first = p * 4 + h * (BK / 16);
  int n = total - first;
  return n <= 0 ? 0 : (n > BK / 16 ? BK / 16 : n);
}

// y = accumulator (32 fp32 TMEM words) + 32 biases from shared memory, by 16-byte loads
__device__ __forceinline__ void add_bias32(const uint32_t (&v)[32], const float* bl, float (&y)[32]) {
  const float4* b4 = reinterpret_cast<const float4*>(bl);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 b = b4[j];
    y[4 * j] = __uint_as_float(v[4 * j]) + b.x;
    y[4 * j + 1] = __uint_as_float(v[4 * j + 1]) + b.y;
    y[4 * j + 2] = __uint_as_float(v[4 * j + 2]) + b.z;
    y[4 * j + 3] = __uint_as_float(v[4 * j + 3]) + b.w;
  }
}

template <class C, int CG>
__device__ __forceinline__ void mlp_stream_body(const TensorMaps& tm, const ChainArgs& args) {
  using T = typename C::T;
  using L = StreamLayout<C, CG>;
  constexpr bool kPair = CG == 2;
  constexpr int NL = C::NL;
  constexpr int kBS = L::kBStages;
  constexpr int kNB = L::kNB;
  constexpr int NH = L::NH;

  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* b_full = bars;          // [8]
  uint64_t* b_empty = bars + 8;     // [8]
  uint64_t* x_full = bars + 16;     // [2]  x ring slots or resident x buffers
  uint64_t* x_empty = bars + 18;    // [2]
  uint64_t* acc_full = bars + 20;   // [2] per output half
  uint64_t* act_ready = bars + 22;  // [2] per output half
  uint64_t* mma_done = bars + 24;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 26);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 27);
  uint64_t* pair_bar = bars + 28;   // [4] the two epilogue warps of each TMEM lane quarter
  float* bias_s = reinterpret_cast<float*>(smem + L::kOffBias);
  float* ln_g = reinterpret_cast<float*>(smem + L::kOffLn);
  float* ln_b = ln_g + C::N(NL - 1);
  float* head_w = reinterpret_cast<float*>(smem + L::kOffHead);  // [N_last][kHeadPad] fp32
  float* head_b = head_w + C::N(NL - 1) * L::kHeadPad;           // [16]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = kPair ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  // work unit: kBM rows per CTA (one tile, or the pair's two tiles of a 256-row unit)
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
      mbar_init(smem_u32(&x_empty[s]), 1);
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(smem_u32(&acc_full[h]), 1);
      mbar_init(smem_u32(&act_ready[h]), L::kEpiWarps * CG);
    }
    mbar_init(smem_u32(mma_done), 1);
    for (int i = 0; i < 4; ++i) mbar_init(smem_u32(&pair_bar[i]), 64);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) prefetch_tmap(&tm.x);
  // Everything above overlaps the previous kernel of the stream. Global memory is touched only
  // after griddepcontrol.wait, except the per-column parameters when the launch marked them safe
  // (pdl_early bit 1), which are staged first.
  const int early = args.pdl_early;
  if ((early & 1) == 0) pdl_wait_prior();
  // fp32 biases, LayerNorm parameters and head weights
  for (int l = 0; l < NL; ++l) {
    const T* b = reinterpret_cast<const T*>(args.bias[l]);
    for (int i = threadIdx.x; i < C::N(l); i += blockDim.x)
      bias_s[L::biasOff(l) + i] = b != nullptr ? Elem<T>::to_f(b[i]) : 0.0f;
  }
  int ident_local = 1;
  if constexpr (L::kLN) {
    const T* g = reinterpret_cast<const T*>(args.gamma);
    const T* b = reinterpret_cast<const T*>(args.beta);
    for (int i = threadIdx.x; i < C::N(NL - 1); i += blockDim.x) {
      ln_g[i] = g != nullptr ? Elem<T>::to_f(g[i]) : 1.0f;
      ln_b[i] = b != nullptr ? Elem<T>::to_f(b[i]) : 0.0f;
      ident_local &= (ln_g[i] == 1.0f && ln_b[i] == 0.0f) ? 1 : 0;
    }
  }
  // gamma == 1 and beta == 0 everywhere: the LayerNorm affine step is the identity
  const bool ln_ident = __syncthreads_and(ident_local) != 0;
  if constexpr (C::TAIL == kTailHead) {
    // head weights [N_last, HEAD_N] (row-major, 16-bit) -> fp32 [N_last][kHeadPad], zero padded
    const T* hw = reinterpret_cast<const T*>(args.head_w);
    const T* hb = reinterpret_cast<const T*>(args.head_b);
    for (int i = threadIdx.x; i < C::N(NL - 1) * L::kHeadPad; i += blockDim.x) {
      const int k = i / L::kHeadPad, o = i % L::kHeadPad;
      head_w[i] = o < C::HEAD_N ? Elem<T>::to_f(hw[k * C::HEAD_N + o]) : 0.0f;
    }
    for (int i = threadIdx.x; i < 16; i += blockDim.x)
      head_b[i] = (i < C::HEAD_N && hb != nullptr) ? Elem<T>::to_f(hb[i]) : 0.0f;
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
  const int num_units = args.num_tiles;  // in units of kBM * CG rows
  // barrier address as seen by the loads / arrivals of this CTA (the leader's in a pair)
  auto leader_bar = [&](const uint64_t* b) -> uint32_t {
    return kPair ? mapa_shared(smem_u32(b), 0) : smem_u32(b);
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    // Stage order per layer mirrors the MMA issue order: K panel p outer for a streamed-x first
    // layer (each x panel serves both output halves), output half outer otherwise.
    if (lane == 0) {
      const uint64_t keep = l2_policy_evict_last();
      const uint64_t stream = l2_policy_evict_first();
      int bs = 0, xs = 0;
      uint32_t bph = 0, xph = 0;
      bool ok = true;
      // weight rows [row, row + kBK) of output half hf of layer l into the next ring slot
      auto stage = [&](int l, int row, int hf) -> bool {
        if (row >= C::K(l)) return true;
        if (!mbar_wait<kPair>(smem_u32(&b_empty[bs]), bph ^ 1, wctx, kDevTimeoutProducer)) return false;
        const int hw = C::N(l) / NH;
        const int hwc = hw / CG;  // columns staged by this CTA
        if (leader) mbar_arrive_expect_tx(smem_u32(&b_full[bs]), (hwc / 64) * L::kBK * 128 * CG);
        const uint32_t dst = smem_u32(smem + L::kOffB + bs * L::kBStageBytes);
        const uint32_t fb = leader_bar(&b_full[bs]);
        // one request: kBK rows x (hwc / 64) column blocks, block after block in shared memory
        const int blk = (hf * hw + static_cast<int>(rank) * hwc) / 64;
        if constexpr (kPair) {
          tma_load_3d_pair(dst, &tm.w[l], fb, 0, row, blk, keep);
        } else {
          tma_load_3d_hint(dst, &tm.w[l], fb, 0, row, blk, keep);
        }
        if (++bs == kBS) { bs = 0; bph ^= 1; }
        return true;
      };
      // one 64-column x panel of this CTA's rows into x slot xs
      auto load_x = [&](int p, int row) {
        if (leader) mbar_arrive_expect_tx(smem_u32(&x_full[xs]), kPanelBytes * CG);
        const uint32_t dst = smem_u32(smem + L::kOffX + xs * kPanelBytes);
        if constexpr (kPair) {
          tma_load_2d_pair(dst, &tm.x, leader_bar(&x_full[xs]), p * kPanel, row, stream);
        } else {
          tma_load_2d_hint(dst, &tm.x, smem_u32(&x_full[xs]), p * kPanel, row, stream);
        }
      };
#pragma unroll 1
      for (int unit = unit0; ok && unit < num_units; unit += units_step) {
        const int row_base = unit * kBM * CG + static_cast<int>(rank) * kBM;
        if constexpr (L::kXRes) {
          if (!mbar_wait<kPair>(smem_u32(&x_empty[xs]), xph ^ 1, wctx, kDevTimeoutProducer)) break;
          if (args.inject != 1) load_x(0, row_base);
          if (++xs == L::kXSlots) { xs = 0; xph ^= 1; }
        }
#pragma unroll 1
        for (int l = 0; ok && l < NL; ++l) {
          if constexpr (L::kSkip2 != 0) {
            if (l == L::kLoadX2Layer) {
              // the second input into the resident x buffer, once x's last reader is done
              if (!mbar_wait<kPair>(smem_u32(&x_empty[xs]), xph ^ 1, wctx, kDevTimeoutProducer)) break;
              if (args.inject != 1) {
                mbar_arrive_expect_tx(smem_u32(&x_full[xs]), kPanelBytes);
                tma_load_2d_hint(smem_u32(smem + L::kOffX + xs * kPanelBytes), &tm.x2,
                                 smem_u32(&x_full[xs]), 0, row_base, stream);
              }
              if (++xs == L::kXSlots) { xs = 0; xph ^= 1; }
            }
          }
          const int panels = (C::K(l) + kPanel - 1) / kPanel;
          if (!L::kXRes && l == 0) {
#pragma unroll 1
            for (int p = 0; ok && p < panels; ++p) {
              if (!mbar_wait<kPair>(smem_u32(&x_empty[xs]), xph ^ 1, wctx, kDevTimeoutProducer)) { ok = false; break; }
              if (args.inject != 1) load_x(p, row_base);
              if (++xs == L::kXSlots) { xs = 0; xph ^= 1; }
              for (int hf = 0; ok && hf < NH; ++hf)
                for (int kh = 0; ok && kh < L::kSub; ++kh) ok = stage(l, p * kPanel + kh * L::kBK, hf);
            }
          } else {
#pragma unroll 1
            for (int hf = 0; ok && hf < NH; ++hf)
#pragma unroll 1
              for (int row = 0; ok && row < C::K(l); row += L::kBK) ok = stage(l, row, hf);
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    // Each layer's output is computed as two column halves with their own commit (acc_full[h]),
    // so the epilogue of half 0 overlaps the MMAs of half 1, and the next layer's first K half
    // (activation panels of half 0) starts as soon as act_ready[0] says they are written.
    // In a CTA pair only the leader issues: 256-row MMAs over both CTAs' A operands and weight
    // halves, commits multicast to the barriers of both CTAs.
    auto commit_any = [&](uint64_t* bar) {
      if constexpr (kPair) mma_commit_pair(smem_u32(bar), 0x3); else mma_commit(smem_u32(bar));
    };
    if (lane == 0 && leader) {
      const uint32_t act_sm = smem_u32(smem + L::kOffAct);
      const uint32_t x_sm = smem_u32(smem + L::kOffX);
      const uint32_t b_sm = smem_u32(smem + L::kOffB);
      int bs = 0, xs = 0;
      uint32_t bph = 0, xph = 0, rph[2] = {0, 0};
      uint32_t lstep = 0;  // layers issued so far (selects the accumulator region with SPLIT_ACT)
      bool first = true, ok = true;
#pragma unroll 1
      for (int unit = unit0; ok && unit < num_units; unit += units_step) {
        const int xcur = xs;  // resident x buffer of this unit
#pragma unroll 1
        for (int l = 0; ok && l < NL; ++l) {
          bool have[2] = {first, first};
          first = false;
          auto need = [&](int h) -> bool {  // previous epilogue half h is done
            if (have[h]) return true;
            if (!mbar_wait<kPair>(smem_u32(&act_ready[h]), rph[h], wctx, kDevTimeoutMma)) return false;
            rph[h] ^= 1;
            have[h] = true;
            tc_fence_after();
            return true;
          };
          if (!need(0)) { ok = false; break; }
          // a layer wider than the previous one (the last layer of the previous tile for l = 0)
          // writes columns the previous epilogue's second half may still be reading
          const int n_prev = l == 0 ? C::N(NL - 1) : C::N(l - 1);
          if (NH == 2 && C::N(l) > n_prev && !need(1)) { ok = false; break; }
          const int panels = (C::K(l) + kPanel - 1) / kPanel;
          const int hw = C::N(l) / NH;
          // activation panels at or beyond hi_p were written by the previous epilogue's half 1
          const int hi_p = (l == 0 || (NH == 1 && !L::kSplit)) ? panels + 1 : C::N(l - 1) / 128;
          const uint32_t dcol = L::kSplit ? (lstep & 1u) * 256u : 0u;
          const int ab_bf16 = (l == 0 || !C::HIDDEN_F16) ? Elem<T>::kIsBf16 : 0;
          const uint32_t idesc = make_idesc_f16(kBM * CG, hw, ab_bf16, 0, 1);
          const bool p_outer = !L::kXRes && l == 0;
          // A operand of panel p (waits for x where needed); 0 on timeout
          auto a_panel = [&](int p) -> uint32_t {
            const bool from_x = (l == 0) || (C::SKIP != 0 && l == C::SKIP && p == panels - 1) ||
                                (L::kSkip2 != 0 && l == L::kSkip2 && p == panels - 1);
            if (!from_x) return act_sm + p * kPanelBytes;
            if constexpr (L::kXRes) {
              return x_sm + xcur * kPanelBytes;
            } else {
              if (!mbar_wait<kPair>(smem_u32(&x_full[xs]), xph, wctx, kDevTimeoutMma)) return 0u;
              tc_fence_after();
              return x_sm + xs * kPanelBytes;
            }
          };
          // the weight stages of K panel p (stages of at most one panel)
          auto issue = [&](uint32_t a_base, int p, int hf) -> bool {
            for (int kh = 0; kh < L::kSub; ++kh) {
              const int ks = ksteps_in<C, L::kBK>(l, p, kh);
              if (ks == 0) continue;
              if (!mbar_wait<kPair>(smem_u32(&b_full[bs]), bph, wctx, kDevTimeoutMma)) return false;
              tc_fence_after();
              const uint32_t bst = b_sm + bs * L::kBStageBytes;
              for (int k = 0; k < ks; ++k) {
                const int kin = kh * (L::kBK / 16) + k;  // 16-wide K step within the 64-column panel
                const uint64_t adesc = make_sdesc_sw128(a_base + kin * 32, 16, 1024);
                const uint64_t bdesc = make_sdesc_sw128(bst + k * 2048, L::kBK * 128, 1024);
                const uint32_t acc = (p == 0 && kh == 0 && k == 0) ? 0u : 1u;
                if constexpr (kPair) {
                  mma_ss_pair(tmem_base + dcol + hf * hw, adesc, bdesc, idesc, acc);
                } else {
                  mma_ss(tmem_base + dcol + hf * hw, adesc, bdesc, idesc, acc);
                }
              }
              commit_any(&b_empty[bs]);
              if (++bs == kBS) { bs = 0; bph ^= 1; }
            }
            return true;
          };
          if (L::kXRes && l == 0) {
            if (!mbar_wait<kPair>(smem_u32(&x_full[xcur]), xph, wctx, kDevTimeoutMma)) { ok = false; break; }
            tc_fence_after();
          }
          if (L::kSkip2 != 0 && l == L::kSkip2) {
            // the second input took the x buffer's next phase
            xph ^= 1;
            if (!mbar_wait<kPair>(smem_u32(&x_full[xcur]), xph, wctx, kDevTimeoutMma)) { ok = false; break; }
            tc_fence_after();
          }
          if (p_outer) {
            if (NH == 2 && !need(1)) { ok = false; break; }
#pragma unroll 1
            for (int p = 0; ok && p < panels; ++p) {
              const uint32_t a = a_panel(p);
              if (a == 0u) { ok = false; break; }
              ok = issue(a, p, 0) && (NH == 1 || issue(a, p, 1));
              commit_any(&x_empty[xs]);
              if (++xs == L::kXSlots) { xs = 0; xph ^= 1; }
            }
            if (!ok) break;
            commit_any(&acc_full[0]);
            if (NH == 2) commit_any(&acc_full[1]);
          } else {
#pragma unroll 1
            for (int hf = 0; ok && hf < NH; ++hf) {
              if (hf == 1 && !need(1)) { ok = false; break; }
              if constexpr (L::kBK < kPanel) {
                // 32-row stages: per K panel (measured faster here than the stage loop below)
#pragma unroll 1
                for (int p = 0; ok && p < panels; ++p) {
                  if (p >= hi_p && !need(1)) { ok = false; break; }
                  const uint32_t a = a_panel(p);
                  if (a == 0u) { ok = false; break; }
                  ok = issue(a, p, hf);
                }
                if (ok) commit_any(&acc_full[hf]);
                continue;
              }
              // stages of kBK weight rows (one or two K panels); each K step takes its A operand
              // from the shared-memory activation panels or the resident x panel (layer 0, and the
              // skip concat's last panel)
              // descriptors advance by address >> 4: +2 per 32-byte K step inside a panel, +1024
              // per 16 KB panel, +128 per 2 KB (16-row) step of a B stage
              const uint64_t act_desc = make_sdesc_sw128(act_sm, 16, 1024);
              const uint64_t x_desc = make_sdesc_sw128(x_sm + xcur * kPanelBytes, 16, 1024);
#pragma unroll 1
              for (int r0 = 0; ok && r0 < C::K(l); r0 += L::kBK) {
                const int ks = (C::K(l) - r0) / 16 < L::kBK / 16 ? (C::K(l) - r0) / 16 : L::kBK / 16;
                if ((r0 + ks * 16 - 1) / kPanel >= hi_p && !need(1)) { ok = false; break; }
                if (!mbar_wait<kPair>(smem_u32(&b_full[bs]), bph, wctx, kDevTimeoutMma)) { ok = false; break; }
                tc_fence_after();
                const uint64_t bdesc0 = make_sdesc_sw128(b_sm + bs * L::kBStageBytes, L::kBK * 128, 1024);
                const uint32_t d_tmem = tmem_base + dcol + hf * hw;
                const int kg0 = r0 >> 4;
                for (int k = 0; k < ks; ++k) {
                  const int kg = kg0 + k;  // 16-wide K step within the layer
                  const int p = kg >> 2;
                  const uint64_t bdesc = bdesc0 + static_cast<uint64_t>(k * 128);
                  const uint32_t acc = (r0 | k) != 0 ? 1u : 0u;
                  const bool from_x = (l == 0) || (C::SKIP != 0 && l == C::SKIP && p == panels - 1) ||
                                      (L::kSkip2 != 0 && l == L::kSkip2 && p == panels - 1);
                  const uint64_t adesc = from_x ? x_desc + static_cast<uint64_t>((kg & 3) * 2)
                                                : act_desc + static_cast<uint64_t>(kg * 2 + p * (1024 - 8));
                  if constexpr (kPair) {
                    mma_ss_pair(d_tmem, adesc, bdesc, idesc, acc);
                  } else {
                    mma_ss(d_tmem, adesc, bdesc, idesc, acc);
                  }
                }
                commit_any(&b_empty[bs]);
                if (++bs == kBS) { bs = 0; bph ^= 1; }
              }
              if (ok) commit_any(&acc_full[hf]);
            }
            if (!ok) break;
          }
          if constexpr (L::kXRes) {
            if (l == L::kLastXLayer || (L::kSkip2 != 0 && l == L::kSkip2)) commit_any(&x_empty[xcur]);
          }
          // with SPLIT_ACT every epilogue releases both halves: consume the second one once per
          // layer even where no K panel needed it, so the barrier phases stay in step
          if (L::kSplit && !need(1)) { ok = false; break; }
          ++lstep;
        }
        if constexpr (L::kXRes) {
          if (++xs == L::kXSlots) { xs = 0; xph ^= 1; }
        }
      }
      // drain: every issued MMA has completed before TMEM can be released
      commit_any(mma_done);
    }
    if (lane == 0) {
      volatile int no_abort = 0;
      WaitCtx drain{args.status, &no_abort, args.timeout_ns};
      mbar_wait<kPair>(smem_u32(mma_done), 0, drain, kDevTimeoutMma);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..9)
    const int q = warp & 3;           // TMEM lane quarter this warp may access
    const int eg = (warp - 2) >> 2;   // chunk group: even (0) or odd (1) 32-column chunks
    const int r = q * 32 + lane;      // row within the tile
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    uint8_t* act = smem + L::kOffAct;
    // output staging: two buffers per warp inside the activation buffer (panels the last layer
    // no longer reads), or one dedicated buffer per warp
    uint8_t* stg = L::kStgInAct ? act + L::kStgPanel0 * kPanelBytes + q * 4096 + eg * 2048
                                : smem + L::kOffStg + (warp - 2) * L::kStageBytes;
    float* xchg = reinterpret_cast<float*>(smem + L::kOffXchg);
    int sb = 0;
    uint32_t acc_ph[2] = {0, 0};
    bool ok = true;
    auto wait_acc = [&](int h) -> bool {
      if (!mbar_wait<kPair>(smem_u32(&acc_full[h]), acc_ph[h], wctx, kDevTimeoutEpilogue)) return false;
      acc_ph[h] ^= 1;
      tc_fence_after();
      return true;
    };
    auto release = [&](int h) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (kPair) mbar_arrive_cluster(leader_bar(&act_ready[h])); else mbar_arrive(smem_u32(&act_ready[h]));
      }
    };
    // barrier of the two warps of this lane quarter (bounded, like every wait here)
    uint32_t pph = 0;
    auto pair_sync = [&]() -> bool {
      mbar_arrive(smem_u32(&pair_bar[q]));
      const bool r = mbar_wait(smem_u32(&pair_bar[q]), pph, wctx, kDevTimeoutEpilogue);
      pph ^= 1;
      return r;
    };
    // stage 32 packed columns of this warp's 32 rows and store them with one TMA box
    auto store_chunk = [&](int c, int row0, const uint32_t (&pk)[16]) {
      uint8_t* s = L::kStgInAct ? stg + sb * kPanelBytes : stg;
      if (lane == 0) {
        if constexpr (L::kStgInAct) bulk_wait_group_read<1>(); else bulk_wait_group_read<0>();
      }
      __syncwarp();
      stage_chunk32(s, lane, pk);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        if (row0 < args.m && c * 32 < L::kOutN) tma_store_2d(&tm.out, smem_u32(s), c * 32, row0);
        bulk_commit_group();
      }
      if constexpr (L::kStgInAct) sb ^= 1;
    };
    uint32_t estep = 0;  // layers drained so far (the accumulator region with SPLIT_ACT)
#pragma unroll 1
    for (int unit = unit0; ok && unit < num_units; unit += units_step) {
      const int row_base = unit * kBM * CG + static_cast<int>(rank) * kBM;
      const int64_t row = static_cast<int64_t>(row_base) + r;
      const int row0 = row_base + q * 32;
#pragma unroll 1
      for (int l = 0; ok && l < NL; ++l) {
        const uint32_t dcol = L::kSplit ? (estep & 1u) * 256u : 0u;
        ++estep;
        const float* bl = bias_s + L::biasOff(l);
        const int act_id = C::ACT(l);
        const int hc = C::N(l) / 32 / NH;  // 32-column chunks per half (even)
        if (l == L::kSide) {
          // side output: bias + activation, stored from registers (16-byte stores of this row's
          // 32-column chunks); the activation buffer keeps the previous layer's output
          if (!wait_acc(0)) { ok = false; break; }
#pragma unroll 1
          for (int c = eg; c < C::N(l) / 32; c += 2) {
            uint32_t v[32];
            tmem_ld32(t_lane + dcol + c * 32, v);
            tmem_wait_ld();
            uint32_t pk[16];
            act_dispatch(act_id, [&](auto actc) {
              constexpr int A = decltype(actc)::value;
#pragma unroll
              for (int i = 0; i < 16; ++i)
                pk[i] = Elem<T>::pack(act_t<A>(__uint_as_float(v[2 * i]) + bl[c * 32 + 2 * i]),
                                      act_t<A>(__uint_as_float(v[2 * i + 1]) + bl[c * 32 + 2 * i + 1]));
            });
            if (row < args.m) {
              uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<T*>(args.out2) + row * C::N(l) + c * 32);
#pragma unroll
              for (int j = 0; j < 4; ++j) dst[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
            }
          }
          release(0);
          release(1);
        } else if (l + 1 < NL) {
          // hidden layer: bias + activation -> 16-bit A operand of the next layer (K-major SW128)
          // Layers >= 1 read their A operand from this same activation buffer: the second half's
          // MMAs of layer l still read layer l-1's activations, so writing layer l's activations
          // waits for both halves (the next layer still starts as soon as half 0 is written).
          if (NH == 2 && l >= 1 && !(wait_acc(0) && wait_acc(1))) { ok = false; break; }
#pragma unroll 1
          for (int hf = 0; hf < NH; ++hf) {
            if ((NH == 1 || l == 0) && !wait_acc(hf)) { ok = false; break; }
            // one 32-column chunk of this row: bias + activation, packed into the A panel
            auto put_chunk = [&](int c, const uint32_t* v) {
              uint8_t* line = act + (c >> 1) * kPanelBytes + r * 128;
              act_dispatch(act_id, [&](auto actc) {
                constexpr int A = decltype(actc)::value;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  uint32_t pk[4];
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    const int i = j * 8 + e * 2;
                    const float2 bb = *reinterpret_cast<const float2*>(bl + c * 32 + i);
                    const float y0 = act_t<A>(__uint_as_float(v[i]) + bb.x);
                    const float y1 = act_t<A>(__uint_as_float(v[i + 1]) + bb.y);
                    pk[e] = C::HIDDEN_F16 ? Elem<__half>::pack(y0, y1) : Elem<T>::pack(y0, y1);
                  }
                  const int chunk = (c & 1) * 4 + j;
                  *reinterpret_cast<uint4*>(line + ((chunk ^ (r & 7)) * 16)) =
                      make_uint4(pk[0], pk[1], pk[2], pk[3]);
                }
              });
            };
            // SPLIT_ACT: the first half of the activation panels is released by each warp right
            // after it has written its last chunk of that half (before any chunk if it has none)
            const int last0 = (hc / 2 - 1 - eg) >= 0 ? (hc / 2 - 1) - ((hc / 2 - 1 - eg) & 1) : -1;
            if (L::kSplit && last0 < 0) release(0);
            // this warp's chunks two at a time (EPI_PAIRS): both TMEM loads behind one wait
#pragma unroll 1
            for (int c = hf * hc + eg; c < (hf + 1) * hc; c += EpiPairs<C>::value ? 4 : 2) {
              const bool two = EpiPairs<C>::value && c + 2 < (hf + 1) * hc;
              uint32_t v[2][32];
              tmem_ld32(t_lane + dcol + c * 32, v[0]);
              if (two) tmem_ld32(t_lane + dcol + (c + 2) * 32, v[1]);
              tmem_wait_ld();
              put_chunk(c, v[0]);
              if (two) put_chunk(c + 2, v[1]);
              if (L::kSplit && (c == last0 || (two && c + 2 == last0))) {  // first half written
                fence_proxy_async_smem();
                release(0);
              }
            }
            fence_proxy_async_smem();
            release(L::kSplit ? 1 : hf);
          }
        } else if constexpr (C::TAIL == kTailHead) {
          // last tensor layer + activation, then the narrow head on CUDA cores: each group forms
          // the partial dot products of its chunks, group 1 hands them to group 0
          constexpr int HP = L::kHeadPad;
          float o[HP];
#pragma unroll
          for (int i = 0; i < HP; ++i) o[i] = 0.0f;
#pragma unroll 1
          for (int hf = 0; hf < NH; ++hf) {
            if (!wait_acc(hf)) { ok = false; break; }
#pragma unroll 1
            for (int c = hf * hc + eg; c < (hf + 1) * hc; c += 2) {
              uint32_t v[32];
              tmem_ld32(t_lane + dcol + c * 32, v);
              tmem_wait_ld();
              act_dispatch(act_id, [&](auto actc) {
                constexpr int A = decltype(actc)::value;
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                  const int k = c * 32 + i;
                  const float y = act_t<A>(__uint_as_float(v[i]) + bl[k]);
                  const float4* w4 = reinterpret_cast<const float4*>(head_w + k * HP);
#pragma unroll
                  for (int o4 = 0; o4 < HP / 4; ++o4) {
                    const float4 w = w4[o4];
                    o[o4 * 4 + 0] = fmaf(y, w.x, o[o4 * 4 + 0]);
                    o[o4 * 4 + 1] = fmaf(y, w.y, o[o4 * 4 + 1]);
                    o[o4 * 4 + 2] = fmaf(y, w.z, o[o4 * 4 + 2]);
                    o[o4 * 4 + 3] = fmaf(y, w.w, o[o4 * 4 + 3]);
                  }
                }
              });
            }
            release(hf);
            if (L::kSplit) release(1);
          }
          if (!ok) break;
          float4* xo = reinterpret_cast<float4*>(xchg + r * HP);
          if (eg == 1) {
#pragma unroll
            for (int o4 = 0; o4 < HP / 4; ++o4)
              xo[o4] = make_float4(o[o4 * 4], o[o4 * 4 + 1], o[o4 * 4 + 2], o[o4 * 4 + 3]);
          }
          if (!pair_sync()) { ok = false; break; }
          if (eg == 0) {
#pragma unroll
            for (int o4 = 0; o4 < HP / 4; ++o4) {
              const float4 p = xo[o4];
              o[o4 * 4 + 0] += p.x;
              o[o4 * 4 + 1] += p.y;
              o[o4 * 4 + 2] += p.z;
              o[o4 * 4 + 3] += p.w;
            }
            if (row < args.m) {
              T* dst = reinterpret_cast<T*>(args.out) + row * C::HEAD_N;
#pragma unroll
              for (int i = 0; i < C::HEAD_N; ++i) {
                const float y = act_t<C::HEAD_ACT>(o[i] + head_b[i]);
                if constexpr (Elem<T>::kIsBf16) dst[i] = __float2bfloat16_rn(y); else dst[i] = __float2half_rn(y);
              }
            }
          }
          if (!pair_sync()) { ok = false; break; }  // the exchange slots are free again
        } else {
          // last layer: optional (residual +) LayerNorm (statistics pass over TMEM), then store via
          // staging. The residual rows are read with 16-byte loads, once per pass.
          auto resid_add = [&](int c, float (&y)[32]) {
            if constexpr (C::TAIL == kTailResidualLN) {
              if (row < args.m) {
                const uint4* src = reinterpret_cast<const uint4*>(
                    reinterpret_cast<const T*>(args.resid) + row * C::N(NL - 1) + c * 32);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const uint4 w = __ldg(src + j);
                  const T* t = reinterpret_cast<const T*>(&w);
#pragma unroll
                  for (int e = 0; e < 8; ++e) y[j * 8 + e] += Elem<T>::to_f(t[e]);
                }
              }
            }
          };
          float mean = 0.f, rstd = 1.f;
          if constexpr (L::kLN) {
            if (!wait_acc(0) || (NH == 2 && !wait_acc(1))) { ok = false; break; }
            // Row statistics without the cancellation of E[y^2] - mean^2: each warp of the pair
            // accumulates sum and sum of squares of (y - k), k = its first value of the row, so
            // its partial mean and M2 = sum (y - mean_w)^2 are exact to rounding; the two
            // halves are combined with the parallel-variance formula (Chan et al., 1979). The
            // result equals the two-pass mean / biased variance of common/layer_norm_v2.cuh:34-62.
            float s = 0.f, sq = 0.f, k = 0.f;
            constexpr int kChunks = C::N(NL - 1) / 32;
#pragma unroll 1
            for (int c = eg; c < kChunks; c += 2) {
              uint32_t v[32];
              tmem_ld32(t_lane + dcol + c * 32, v);
              tmem_wait_ld();
              float y[32];
              add_bias32(v, bl + c * 32, y);
              resid_add(c, y);
              if (c == eg) k = y[0];
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const float d = y[i] - k;
                s += d;
                sq = fmaf(d, d, sq);
              }
            }
            const float n_me = 32.0f * ((kChunks - eg + 1) / 2);
            const float mean_me = k + s / n_me;
            const float m2_me = fmaxf(sq - s * (s / n_me), 0.0f);
            float2* xs = reinterpret_cast<float2*>(xchg);
            xs[eg * kBM + r] = make_float2(mean_me, m2_me);
            if (!pair_sync()) { ok = false; break; }
            const float2 other = xs[(eg ^ 1) * kBM + r];
            if (!pair_sync()) { ok = false; break; }  // the exchange slots are free again
            // evaluate in warp order (even half first) so that both warps get identical bits
            const float2 h0 = eg == 0 ? make_float2(mean_me, m2_me) : other;
            const float2 h1 = eg == 0 ? other : make_float2(mean_me, m2_me);
            const float n0 = 32.0f * ((kChunks + 1) / 2), n1 = 32.0f * (kChunks / 2);
            const float inv_n = 1.0f / C::N(l);
            mean = (h0.x * n0 + h1.x * n1) * inv_n;
            const float delta = h1.x - h0.x;
            const float var = (h0.y + h1.y + delta * delta * (n0 * n1 * inv_n)) * inv_n;
            rstd = rsqrtf(var + args.ln_eps);
          }
#pragma unroll 1
          for (int hf = 0; hf < NH; ++hf) {
            if constexpr (!L::kLN) {
              if (!wait_acc(hf)) { ok = false; break; }
            }
#pragma unroll 1
            for (int c = hf * hc + eg; c < (hf + 1) * hc; c += 2) {
              uint32_t v[32];
              tmem_ld32(t_lane + dcol + c * 32, v);
              tmem_wait_ld();
              if (c + 2 >= (hf + 1) * hc) release(hf);  // this warp's part of the half is read
              uint32_t pk[16];
              float yr[32];
              add_bias32(v, bl + c * 32, yr);
              resid_add(c, yr);
              if constexpr (L::kLN) {
                const float nmr = -mean * rstd;
                if (ln_ident) {
#pragma unroll
                  for (int i = 0; i < 16; ++i)
                    pk[i] = Elem<T>::pack(fmaf(yr[2 * i], rstd, nmr), fmaf(yr[2 * i + 1], rstd, nmr));
                } else {
                  const float4* g4 = reinterpret_cast<const float4*>(ln_g + c * 32);
                  const float4* b4 = reinterpret_cast<const float4*>(ln_b + c * 32);
#pragma unroll
                  for (int j = 0; j < 8; ++j) {
                    const float4 g = g4[j], b = b4[j];
                    pk[2 * j] = Elem<T>::pack(fmaf(fmaf(yr[4 * j], rstd, nmr), g.x, b.x),
                                              fmaf(fmaf(yr[4 * j + 1], rstd, nmr), g.y, b.y));
                    pk[2 * j + 1] = Elem<T>::pack(fmaf(fmaf(yr[4 * j + 2], rstd, nmr), g.z, b.z),
                                                  fmaf(fmaf(yr[4 * j + 3], rstd, nmr), g.w, b.w));
                  }
                }
              } else {
                act_dispatch(act_id, [&](auto actc) {
                  constexpr int A = decltype(actc)::value;
#pragma unroll
                  for (int i = 0; i < 16; ++i) pk[i] = Elem<T>::pack(act_t<A>(yr[2 * i]), act_t<A>(yr[2 * i + 1]));
                });
              }
              store_chunk(c, row0, pk);
            }
          }
          if (L::kSplit) release(1);
          if constexpr (L::kStgInAct) {
            // the next tile's hidden epilogue rewrites this lane quarter of the activation
            // buffer: both warps' stores must have read their staging first
            if (lane == 0) bulk_wait_group_read<0>();
            __syncwarp();
            if (!pair_sync()) { ok = false; break; }
          }
        }
      }
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
    mlp_stream_kernel(const __grid_constant__ TensorMaps tm, const ChainArgs args) {
  mlp_stream_body<C, 1>(tm, args);
}

// CTA-pair form: two CTAs of a cluster share each weight stage (half of its columns each).
template <class C>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(320, 1)
    mlp_stream_pair_kernel(const __grid_constant__ TensorMaps tm, const ChainArgs args) {
  mlp_stream_body<C, 2>(tm, args);
}

}  // namespace gp
