// Instantiations of the weight-streaming chain kernel (wide layers).
#include <type_traits>

#include "stream_launch.cuh"

namespace gp {

// DLRM bottom MLP (common/mlps.py:23-35 DlrmMlp([K0, 512, 256, 128])): K0 = 16 is BASELINE's
// 13 dense features padded to 16; K0 = 32 is the reference app's own width
// (apps/dlrm_botmlp/pipelined/val.py:11-12, DlrmMlp([13 + 19, 512, 256, 128]), x [M, 32]).
template <int K0_>
struct ChainDlrmBot {
  using T = __half;
  static constexpr int NL = 3;
  __host__ __device__ static constexpr int K(int l) { return l == 0 ? K0_ : (l == 1 ? 512 : 256); }
  __host__ __device__ static constexpr int N(int l) { return l == 0 ? 512 : (l == 1 ? 256 : 128); }
  __host__ __device__ static constexpr int ACT(int) { return kActRelu; }
  static constexpr int SKIP = 0, TAIL = kTailNone, HEAD_N = 0, HEAD_ACT = kActNone;
  static constexpr bool HIDDEN_F16 = false;
  static constexpr int HALVES = 2;
  static constexpr bool SPLIT_ACT = false;
  static constexpr bool EPI_PAIRS = false;
};

// GraphCast-style edge / node MLP (apps/gc_edges/torch/model.py:4-14): K0 -> 512 act -> 512, LN.
template <typename TT, int K0_, int ACT0>
struct ChainGc {
  using T = TT;
  static constexpr int NL = 2;
  __host__ __device__ static constexpr int K(int l) { return l == 0 ? K0_ : 512; }
  __host__ __device__ static constexpr int N(int) { return 512; }
  __host__ __device__ static constexpr int ACT(int l) { return l == 0 ? ACT0 : kActNone; }
  static constexpr int SKIP = 0, TAIL = kTailLayerNorm, HEAD_N = 0, HEAD_ACT = kActNone;
  static constexpr bool HIDDEN_F16 = std::is_same<TT, __nv_bfloat16>::value;
  static constexpr int HALVES = 2;
  static constexpr bool SPLIT_ACT = false;
};

// NeRF trunk without view directions (apps/nerf_full/torch/model.py:5-66, use_viewdirs=False):
// 63(64) -> 256 x5 (ReLU), concat x -> 319(320) -> 256, 256 -> 256 x2 (ReLU), decode 256 -> 4.
struct ChainNerf {
  using T = __half;
  static constexpr int NL = 8;
  __host__ __device__ static constexpr int K(int l) { return l == 0 ? 64 : (l == 5 ? 320 : 256); }
  __host__ __device__ static constexpr int N(int) { return 256; }
  __host__ __device__ static constexpr int ACT(int) { return kActRelu; }
  static constexpr int SKIP = 5, TAIL = kTailHead, HEAD_N = 4, HEAD_ACT = kActNone;
  static constexpr bool HIDDEN_F16 = false;
  static constexpr int HALVES = 1;
  static constexpr bool SPLIT_ACT = true;
};

// The same trunk without the head: layer 8's ReLU output is the result (apps/nerf_a).
struct ChainNerfTrunk : ChainNerf {
  static constexpr int TAIL = kTailNone, HEAD_N = 0;
};

// BERT attention-output block (apps/bert_addln_ffn/torch/model.py:4-19, H = 128, ff = 512):
//   stage 1: h = LN0(attn_out W0 + b0 + x)        -- one 128-wide layer, residual x
//   stage 2: y = LN2(ReLU(h W1 + b1) W2 + b2 + h)  -- 128 -> 512 -> 128, residual h
struct ChainAddLn0 {
  using T = __half;
  static constexpr int NL = 1;
  __host__ __device__ static constexpr int K(int) { return 128; }
  __host__ __device__ static constexpr int N(int) { return 128; }
  __host__ __device__ static constexpr int ACT(int) { return kActNone; }
  static constexpr int SKIP = 0, TAIL = kTailResidualLN, HEAD_N = 0, HEAD_ACT = kActNone;
  static constexpr bool HIDDEN_F16 = false;
  static constexpr int HALVES = 1;
  static constexpr bool SPLIT_ACT = false;
};

// The FFN stage is also the reference's own small BERT FFN (apps/bert_ffn, 128 -> 512 ReLU -> 128,
// + x, LN): fp16, and bf16 with fp16 hidden activations.
template <typename TT>
struct ChainFfnResLn {
  using T = TT;
  static constexpr int NL = 2;
  __host__ __device__ static constexpr int K(int l) { return l == 0 ? 128 : 512; }
  __host__ __device__ static constexpr int N(int l) { return l == 0 ? 512 : 128; }
  __host__ __device__ static constexpr int ACT(int l) { return l == 0 ? kActRelu : kActNone; }
  static constexpr int SKIP = 0, TAIL = kTailResidualLN, HEAD_N = 0, HEAD_ACT = kActNone;
  static constexpr bool HIDDEN_F16 = std::is_same<TT, __nv_bfloat16>::value;
  static constexpr int HALVES = 2;
  static constexpr bool SPLIT_ACT = false;
};

int launch_addln0_f16_h128(const LaunchCtx& c) { return launch_stream<ChainAddLn0>(c); }
int launch_ffn_resln_f16_h128(const LaunchCtx& c) { return launch_stream<ChainFfnResLn<__half>>(c); }
int launch_ffn_resln_bf16_h128(const LaunchCtx& c) {
  return launch_stream<ChainFfnResLn<__nv_bfloat16>>(c);
}

// NeRF with view directions (apps/nerf_full/torch/model.py:40-64 with use_viewdirs=True; the
// reference's pipelined shapes, nerf_full_pl_ext.cu:24-68): x [M, 64], d [M, 32]; one fused
// chain of twelve tensor-core layers per 128-row tile:
//   0..7   the trunk (w1..w8; w6 [320, 256] reads [h | x])                      -> encoded
//   8      alpha = encoded w9 + b9 ([256, 64]), a side output stored to out_r; the activation
//          buffer keeps `encoded`
//   9      bottleneck = encoded w10 + b10 ([256, 256])
//   10     ReLU([bottleneck | d] w11 + b11): w11 [288, 128] read as 320 rows (rows 288..319 are
//          past the tensor and read as zeros), d the second input, zero filled to 64 columns
//   11     w12 + b12 ([128, 64])                                                  -> out_rgb
// No intermediate leaves the SM: `encoded`, the bottleneck and the rgb hidden layer stay in
// the activation buffer, and d is loaded into the resident x buffer after the skip layer.
struct ChainNerfFull {
  using T = __half;
  static constexpr int NL = 12;
  __host__ __device__ static constexpr int K(int l) {
    return l == 0 ? 64 : (l == 5 || l == 10) ? 320 : (l == 11 ? 128 : 256);
  }
  __host__ __device__ static constexpr int N(int l) {
    return l < 8 ? 256 : (l == 8 || l == 11) ? 64 : (l == 9 ? 256 : 128);
  }
  __host__ __device__ static constexpr int ACT(int l) {
    return (l < 8 || l == 10) ? kActRelu : kActNone;
  }
  __host__ __device__ static constexpr int WROWS(int l) { return l == 10 ? 288 : K(l); }
  static constexpr int SKIP = 5, TAIL = kTailNone, HEAD_N = 0, HEAD_ACT = kActNone;
  static constexpr int SIDE = 8, SKIP2 = 10, X2_COLS = 32;
  static constexpr bool HIDDEN_F16 = false;
  static constexpr int HALVES = 1;
  static constexpr bool SPLIT_ACT = true;
};

int launch_nerf_full(const LaunchCtx& base, int64_t m, const void* x, const void* d,
                     const void* const* w, const void* const* b, void* out_r, void* out_rgb) {
  gp_mlp_spec spec{};
  spec.dtype = GP_F16;
  LaunchCtx t = base;
  t.spec = &spec;
  t.m = m;
  t.x = x;
  t.x2 = d;
  t.x_ld = 0;
  t.out = out_rgb;
  t.out_ld = 0;
  for (int l = 0; l < ChainNerfFull::NL; ++l) {
    t.w[l] = w[l];
    t.args.bias[l] = b[l];
  }
  t.args.m = m;
  t.args.num_tiles = static_cast<int>((m + kBM - 1) / kBM);
  t.args.out = out_rgb;
  t.args.out2 = out_r;
  return launch_stream<ChainNerfFull>(t);
}

int launch_dlrm_bot_f16(const LaunchCtx& c) { return launch_stream<ChainDlrmBot<16>>(c); }
int launch_dlrm_bot_f16_k32(const LaunchCtx& c) { return launch_stream<ChainDlrmBot<32>>(c); }
int launch_gc_silu_bf16_k1536(const LaunchCtx& c) { return launch_stream<ChainGc<__nv_bfloat16, 1536, kActSilu>, 2>(c); }
int launch_gc_relu_bf16_k1536(const LaunchCtx& c) { return launch_stream<ChainGc<__nv_bfloat16, 1536, kActRelu>, 2>(c); }
int launch_gc_relu_f16_k1536(const LaunchCtx& c) { return launch_stream<ChainGc<__half, 1536, kActRelu>, 2>(c); }
int launch_gc_relu_f16_k1024(const LaunchCtx& c) { return launch_stream<ChainGc<__half, 1024, kActRelu>, 2>(c); }
int launch_nerf_f16(const LaunchCtx& c) { return launch_stream<ChainNerf>(c); }
int launch_nerf_trunk_f16(const LaunchCtx& c) { return launch_stream<ChainNerfTrunk>(c); }

}  // namespace gp
