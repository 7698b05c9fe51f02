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

// NeRF with view directions (apps/nerf_full, model.py:40-64 with use_viewdirs=True; the
// reference's pipelined shapes, nerf_full_pl_ext.cu:24-68): x [M, 64], d [M, 32]; trunk w1..w8
// (w6 [320, 256] reads [h | x]); alpha w9 [256, 64]; bottleneck w10 [256, 256];
// rgb w11 [288, 128] reads [bottleneck | d], w12 [128, 64]. Three chain launches:
//   trunk  x -> encoded, stored in columns 0..255 of a [M, 384] buffer E
//   alpha  encoded (E, row stride 384) -> out_r [M, 64]
//   rgb    E = [encoded | d | 0] (384) -> 384 -> 128 (ReLU) -> 128, of which the first 64
//          columns are stored to out_rgb
// The rgb chain's first layer carries the bottleneck in its first 256 columns and a 32 x 32
// identity that passes d through unchanged (x 1.0, exact) to columns 256..287, so the concat
// [bottleneck | d] is simply its output; w11 is zero-padded to 384 rows, w12 to 128 columns.
struct ChainNerfAlpha {
  using T = __half;
  static constexpr int NL = 1;
  __host__ __device__ static constexpr int K(int) { return 256; }
  __host__ __device__ static constexpr int N(int) { return 64; }
  __host__ __device__ static constexpr int ACT(int) { return kActNone; }
  static constexpr int SKIP = 0, TAIL = kTailNone, HEAD_N = 0, HEAD_ACT = kActNone;
  static constexpr bool HIDDEN_F16 = false;
  static constexpr int HALVES = 1;
  static constexpr bool SPLIT_ACT = false;
};

struct ChainNerfRgb {
  using T = __half;
  static constexpr int NL = 3;
  __host__ __device__ static constexpr int K(int l) { return l == 2 ? 128 : 384; }
  __host__ __device__ static constexpr int N(int l) { return l == 0 ? 384 : 128; }
  __host__ __device__ static constexpr int ACT(int l) { return l == 1 ? kActRelu : kActNone; }
  static constexpr int SKIP = 0, TAIL = kTailNone, HEAD_N = 0, HEAD_ACT = kActNone;
  static constexpr bool HIDDEN_F16 = false;
  static constexpr int HALVES = 2;
  static constexpr bool SPLIT_ACT = false;
  static constexpr int OUT_N = 64;
};

// E[:, 256:384] = [d | 0] with 16-byte loads and stores (16 per row: 4 carry d, 12 zeros).
__global__ void nerf_stage_d_kernel(const uint4* __restrict__ d, uint4* __restrict__ e, int64_t m) {
  const int64_t n = m * 16;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i >> 4;
    const int c = static_cast<int>(i & 15);
    e[row * 48 + 32 + c] = c < 4 ? __ldg(d + row * 4 + c) : make_uint4(0, 0, 0, 0);
  }
}

__global__ void nerf_identity_block_kernel(__half* w0p) {  // w0p [384, 384]: 1.0 at (256 + i, 256 + i)
  const int i = threadIdx.x;
  if (i < 32) w0p[(256 + i) * 384 + 256 + i] = __float2half_rn(1.0f);
}

int launch_nerf_full(const LaunchCtx& base, int64_t m, const void* x, const void* d,
                     const void* const* w, const void* const* b, void* out_r, void* out_rgb) {
  auto al = [](size_t v) { return (v + 255) / 256 * 256; };
  const size_t e_bytes = al(size_t(m) * 384 * 2), w0_bytes = al(384 * 384 * 2), b0_bytes = al(384 * 2);
  const size_t w1_bytes = al(384 * 128 * 2), w2_bytes = al(128 * 128 * 2), b2_bytes = al(128 * 2);
  void* ws = nullptr;
  const cudaStream_t s = base.stream;
  int rc = workspace_acquire(e_bytes + w0_bytes + b0_bytes + w1_bytes + w2_bytes + b2_bytes, s, &ws);
  if (rc != GP_OK) return rc;
  char* p = static_cast<char*>(ws);
  __half* E = reinterpret_cast<__half*>(p);
  char* w0p = p + e_bytes;
  char* b0p = w0p + w0_bytes;
  char* w1p = b0p + b0_bytes;
  char* w2p = w1p + w1_bytes;
  char* b2p = w2p + w2_bytes;
  cudaError_t e = cudaSuccess;
  auto ck = [&](cudaError_t r) { if (e == cudaSuccess) e = r; };
  // augmented weights of the rgb chain
  ck(cudaMemsetAsync(w0p, 0, w0_bytes + b0_bytes + w1_bytes + w2_bytes + b2_bytes, s));
  ck(cudaMemcpy2DAsync(w0p, 384 * 2, w[9], 256 * 2, 256 * 2, 256, cudaMemcpyDeviceToDevice, s));
  nerf_identity_block_kernel<<<1, 32, 0, s>>>(reinterpret_cast<__half*>(w0p));
  if (b[9] != nullptr) ck(cudaMemcpyAsync(b0p, b[9], 256 * 2, cudaMemcpyDeviceToDevice, s));
  ck(cudaMemcpyAsync(w1p, w[10], 288 * 128 * 2, cudaMemcpyDeviceToDevice, s));
  ck(cudaMemcpy2DAsync(w2p, 128 * 2, w[11], 64 * 2, 64 * 2, 128, cudaMemcpyDeviceToDevice, s));
  if (b[11] != nullptr) ck(cudaMemcpyAsync(b2p, b[11], 64 * 2, cudaMemcpyDeviceToDevice, s));
  // E = [encoded | d | 0]: d into columns 256..287, zeros into 288..383 (encoded by the trunk)
  {
    const int64_t want = (m * 16 + 255) / 256;
    const int blocks = static_cast<int>(want < 8 * base.sm_count ? want : 8 * base.sm_count);
    nerf_stage_d_kernel<<<blocks, 256, 0, s>>>(static_cast<const uint4*>(d), reinterpret_cast<uint4*>(E), m);
  }
  if (e != cudaSuccess) rc = set_error(GP_ERR_CUDA, "nerf_full staging: %s", cudaGetErrorString(e));

  gp_mlp_spec spec{};
  spec.dtype = GP_F16;
  LaunchCtx t = base;
  t.spec = &spec;
  t.m = m;
  t.args.m = m;
  t.args.num_tiles = static_cast<int>((m + kBM - 1) / kBM);
  for (int l = 0; l < kMaxLayers; ++l) t.args.bias[l] = nullptr;
  if (rc == GP_OK) {  // trunk: x -> E[:, 0:256]
    t.x = x;
    t.x_ld = 0;
    t.out = E;
    t.out_ld = 384;
    for (int l = 0; l < 8; ++l) {
      t.w[l] = w[l];
      t.args.bias[l] = b[l];
    }
    t.args.out = t.out;
    rc = launch_stream<ChainNerfTrunk>(t);
  }
  if (rc == GP_OK) {  // alpha: encoded -> out_r
    t.x = E;
    t.x_ld = 384;
    t.out = out_r;
    t.out_ld = 0;
    t.w[0] = w[8];
    t.args.bias[0] = b[8];
    t.args.out = t.out;
    rc = launch_stream<ChainNerfAlpha>(t);
  }
  if (rc == GP_OK) {  // rgb: [encoded | d | 0] -> out_rgb
    t.x = E;
    t.x_ld = 0;
    t.out = out_rgb;
    t.w[0] = w0p;
    t.w[1] = w1p;
    t.w[2] = w2p;
    t.args.bias[0] = b0p;
    t.args.bias[1] = b[10];
    t.args.bias[2] = b2p;
    t.args.out = t.out;
    rc = launch_stream<ChainNerfRgb>(t);
  }
  workspace_release(s);
  return rc;
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
