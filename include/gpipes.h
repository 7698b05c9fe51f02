/*
 * gpipes.h -- C ABI of the B200 fused-MLP library (libgpipes.so).
 *
 * Each gp_<app>_out entry point replaces one reference launch function: same argument order
 * (x, then w_i, b_i per layer, then LayerNorm gamma/beta, then out), all caller-owned device
 * pointers, plus the row count and the caller's CUDA stream. The reference binds these through
 * pybind11 (`cuda_ext.<app>_out`); a ctypes / cgo / JNI binding of this header is a drop-in.
 *
 * Conventions (shared by every entry point):
 *   - x     [m, K0]        row-major, 16-bit (fp16 unless the entry point takes a dtype)
 *   - w_l   [K_l, N_l]     row-major, i.e. the transpose of torch.nn.Linear.weight, exactly as the
 *                          reference passes `weight.t().contiguous()`
 *                          (apps/mgn_fullmlp/pipelined/val.py:17-19)
 *   - b_l   [N_l]          16-bit; NULL means "no bias"
 *   - gamma, beta [N_last] 16-bit LayerNorm affine parameters; NULL means 1 / 0
 *   - out   [m, N_last]    row-major, 16-bit, written completely
 *   - x, w_l and out must be 16-byte aligned and their row pitch a multiple of 16 bytes;
 *     b_l, gamma, beta must be 4-byte aligned.
 *   - stream is a cudaStream_t (NULL = legacy default stream). Calls are asynchronous.
 *   - Accumulation is fp32; hidden activations are rounded to the 16-bit input type.
 *   - m may be 0 (no-op) and need not be a multiple of the 128-row tile.
 *
 * Return value: GP_OK or a negative gp_status; gp_last_error() gives a message (thread-local).
 * Device-side timeouts (a bounded wait that ran out) are reported asynchronously through
 * gp_device_status(); with the environment variable GP_SYNC_CHECK=1 every call synchronises its
 * stream and returns GP_ERR_TIMEOUT itself.
 */
#ifndef GPIPES_H_
#define GPIPES_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GP_MAX_LAYERS 10

#if defined(__GNUC__)
#define GP_API __attribute__((visibility("default")))
#else
#define GP_API
#endif

typedef enum gp_status {
  GP_OK = 0,
  GP_ERR_ARG = -1,          /* null pointer or negative size */
  GP_ERR_SHAPE = -2,        /* widths do not match the entry point */
  GP_ERR_ALIGN = -3,        /* pointer or pitch violates the alignment rules above */
  GP_ERR_UNSUPPORTED = -4,  /* no compiled kernel for this layer chain */
  GP_ERR_CUDA = -5,         /* CUDA runtime / launch error */
  GP_ERR_TIMEOUT = -6,      /* a device-side bounded wait ran out (kernel aborted cleanly) */
  GP_ERR_DRIVER = -7        /* TMA descriptor creation failed */
} gp_status;

typedef enum gp_dtype { GP_F16 = 0, GP_BF16 = 1 } gp_dtype;

typedef enum gp_act {
  GP_ACT_NONE = 0,
  GP_ACT_RELU = 1,
  GP_ACT_GELU_TANH = 2,
  GP_ACT_SILU = 3,
  GP_ACT_SIGMOID = 4
} gp_act;

typedef enum gp_tail {
  GP_TAIL_NONE = 0,         /* out = act_last(x_L W_L + b_L) */
  GP_TAIL_LAYERNORM = 1,    /* out = LN(x_L W_L + b_L) */
  GP_TAIL_RESIDUAL_LN = 2   /* out = LN(x_L W_L + b_L + x) (BERT FFN) */
} gp_tail;

/* A layer chain. widths[0] is the stored (padded) input width K0; layer l maps widths[l] to
 * widths[l+1] and applies act[l] (the last layer's act is ignored when tail is a LayerNorm).
 * skip_layer = s > 0 makes layer s read the concatenation [output of layer s-1 || x] (the NeRF
 * skip connection); its weight is then [widths[s] + widths[0], widths[s+1]]. 0 = no skip. */
typedef struct gp_mlp_spec {
  int n_layers;
  int widths[GP_MAX_LAYERS + 1];
  int act[GP_MAX_LAYERS];
  int tail;         /* gp_tail */
  int dtype;        /* gp_dtype */
  float ln_eps;
  int skip_layer;
} gp_mlp_spec;

/* ---------------------------------------------------------------------------------------------
 * Generic entry point: any chain for which a kernel is compiled (the per-app functions below
 * wrap it). No reference counterpart (the reference fixes one chain per app at compile time).
 * ------------------------------------------------------------------------------------------- */
GP_API int gp_fused_mlp_out(const gp_mlp_spec* spec, int64_t m, const void* x,
                     const void* const* w, const void* const* b,
                     const void* gamma, const void* beta, void* out, void* stream);

/* MeshGraphNet MLP + LayerNorm, fp16, eps 1e-5.
 * Replaces mgn_fullmlp_out (apps/mgn_fullmlp/pipelined/mgn_fullmlp_pl_ext.cu:24-71), which fixes
 * k0 = 384; k0 = 256 is the MeshGraphNet node MLP, k0 = 128 also accepted.
 * Chain: k0 -> 128 (ReLU) -> 128 (ReLU) -> 128, LayerNorm(128). */
GP_API int gp_mgn_fullmlp_out(int64_t m, int k0, const void* x,
                       const void* w1, const void* b1, const void* w2, const void* b2,
                       const void* w3, const void* b3, const void* gamma, const void* beta,
                       void* out, void* stream);

/* Same chain without the LayerNorm.
 * Replaces mgn_linears_out (apps/mgn_linears/pipelined/mgn_linears_pl_ext.cu:24-66). */
GP_API int gp_mgn_linears_out(int64_t m, int k0, const void* x,
                       const void* w1, const void* b1, const void* w2, const void* b2,
                       const void* w3, const void* b3, void* out, void* stream);

/* 128 -> 128 (ReLU) -> 128 (ReLU) -> 128, fp16.
 * Replaces testmlp_out (apps/test_mlp/pipelined/test_mlp_pl_ext.cu:37-82). */
GP_API int gp_testmlp_out(int64_t m, const void* x,
                   const void* w1, const void* b1, const void* w2, const void* b2,
                   const void* w3, const void* b3, void* out, void* stream);

/* DLRM bottom MLP, fp16: x [m, k0] -> 512 -> 256 -> 128, ReLU after every layer; w1 is [k0, 512].
 * k0 = 32 is the reference app's input (apps/dlrm_botmlp/pipelined/val.py:11-12,
 * DlrmMlp([13 + 19, 512, 256, 128])); k0 = 16 is 13 dense features zero padded to 16 (rows
 * 13..15 of w1 multiply the padding). Other widths return GP_ERR_UNSUPPORTED.
 * Replaces dlrm_botmlp_out (apps/dlrm_botmlp/pipelined/dlrm_botmlp_pl_ext.cu:24-66), whose
 * widths are compile-time; here k0 is an argument, as in gp_mgn_fullmlp_out. */
GP_API int gp_dlrm_botmlp_out(int64_t m, int k0, const void* x,
                       const void* w1, const void* b1, const void* w2, const void* b2,
                       const void* w3, const void* b3, void* out, void* stream);

/* GraphCast edge MLP: x [m, 1536] -> 512 (act) -> 512, LayerNorm(512, eps 1e-5).
 * Replaces gc_edges_out (apps/gc_edges/pipelined/gc_edges_pl_ext.cu:24-57), which is fp16 with
 * ReLU; dtype (GP_F16 / GP_BF16) and act (GP_ACT_RELU / GP_ACT_SILU) select the variant. */
GP_API int gp_gc_edges_out(int64_t m, int dtype, int act, const void* x,
                    const void* w0, const void* b0, const void* w1, const void* b1,
                    const void* gamma, const void* beta, void* out, void* stream);

/* GraphCast node MLP: as gp_gc_edges_out with x [m, 1024].
 * Replaces gc_nodes_out (apps/gc_nodes/pipelined/gc_nodes_pl_ext.cu:24-57). */
GP_API int gp_gc_nodes_out(int64_t m, int dtype, int act, const void* x,
                    const void* w0, const void* b0, const void* w1, const void* b1,
                    const void* gamma, const void* beta, void* out, void* stream);

/* BERT-large FFN with residual and LayerNorm, bf16: out = LN(x + W2 gelu_tanh(W1 x + b1) + b2),
 * x [m, 1024], w1 [1024, 4096], w2 [4096, 1024], LN(1024, ln_eps) with gamma/beta.
 * Replaces bert_ffn_out (apps/bert_ffn/pipelined/bert_ffn_pl_ext.cu:24-57), whose app is the
 * 128 -> 512 (ReLU) -> 128 fp16 block; this entry point runs the BERT-large widths. */
GP_API int gp_bert_ffn_out(int64_t m, const void* x, const void* w1, const void* b1,
                    const void* w2, const void* b2, const void* gamma, const void* beta,
                    float ln_eps, void* out, void* stream);

/* DLRM feature interaction between the bottom and top MLPs (graphmodel/dlrm.py:28-42, where it
 * is the `interact_bmm` + `interact_index` + concat nodes; the reference has no kernel for it).
 * For each of the m samples, F = [bot; e_0 .. e_25] (27 x 128) with bot [m, 128] the bottom MLP
 * output and sparse [m, 26, 128] the embedding vectors; out [m, 480] = [bot | Z[a][b], a > b,
 * row-major over the strict lower triangle of Z = F F^T (351 values) | 0]: the top MLP's input.
 * fp16, fp32 accumulation. */
GP_API int gp_dlrm_interaction_out(int64_t m, const void* bot, const void* sparse, void* out,
                                   void* stream);

/* BERT attention-output block at the reference's widths (H = 128, ff = 512, fp16, ReLU, LN eps
 * 1e-5): out = LN2(ReLU(h W1 + b1) W2 + b2 + h) with h = LN0(attn_out W0 + b0 + x).
 * Replaces apps/bert_addln_ffn/pipelined/bert_addln_ffn_pl_ext.cu:15-58 bert_addln_ffn_out
 * (same argument order). attn_out, x, out: [m, 128]; w0 [128, 128], w1 [128, 512], w2 [512, 128];
 * b*, ga*, be*: [N]. Runs as two fused chains with h in a per-device workspace. */
GP_API int gp_bert_addln_ffn_out(int64_t m, const void* attn_out, const void* x, const void* w0,
                                 const void* b0, const void* w1, const void* b1, const void* w2,
                                 const void* b2, const void* ga0, const void* be0, const void* ga2,
                                 const void* be2, void* out, void* stream);

/* DLRM top MLP, fp16, w[5], b[5], two compiled width sets:
 *   k0 = 512, n_out = 64: the reference app's own model (apps/dlrm_topmlp/pipelined/val.py:11-12,
 *     DlrmMlp([479 + 33, 1024, 1024, 512, 256, 64])): 512 -> 1024 -> 1024 -> 512 -> 256 -> 64,
 *     ReLU after every layer, out [m, 64];
 *   k0 = 480, n_out = 1: 479 interaction features zero padded to 480, 480 -> 1024 -> 1024 -> 512
 *     -> 256 (ReLU) -> 1 with a sigmoid (DlrmMlp(..., sigmoid_i=4)), out [m, 1].
 * Other widths return GP_ERR_UNSUPPORTED.
 * Replaces dlrm_topmlp_out (apps/dlrm_topmlp/pipelined/dlrm_topmlp_pl_ext.cu:24-71). */
GP_API int gp_dlrm_topmlp_out(int64_t m, int k0, int n_out, const void* x, const void* const* w,
                       const void* const* b, void* out, void* stream);

/* NeRF trunk, fp16: x [m, 64] (63 positional-encoding features, zero padded); layers 1-5
 * 64 -> 256 -> ... -> 256 (ReLU), layer 6 reads [h || x] (w6 is [320, 256]), layers 7-8
 * 256 -> 256 (ReLU); out [m, 256].
 * Replaces nerf_a_out (apps/nerf_a/pipelined/nerf_a_pl_ext.cu:24-77); w[8], b[8] = layers 1..8. */
GP_API int gp_nerf_a_out(int64_t m, const void* x, const void* const* w, const void* const* b,
                  void* out, void* stream);

/* NeRF MLP with its output head (apps/nerf_full/torch/model.py:5-66, use_viewdirs = False):
 * the trunk of gp_nerf_a_out followed by decode 256 -> 4 (no activation); out [m, 4].
 * w[9], b[9] = layers 1..8 and the head (w[8] is [256, 4]). No reference launch function (the
 * reference's pipelined NeRF kernels stop at the trunk or add the view-direction heads). */
GP_API int gp_nerf_out(int64_t m, const void* x, const void* const* w, const void* const* b,
                void* out, void* stream);

/* MeshGraphNet edge update with the gather and the aggregation fused (graphmodel/mgn_dp.py:28-32
 * update_edges, with the MLP of common/mlps.py MgnMlp(384, [128, 128, 128]); the aggregation is
 * graphmodel/common.py:97-99 UnsortedSegmentSum by destination node). No reference kernel: the
 * reference's mgn_fullmlp_out takes the concatenated [m, 384] rows, built beforehand in HBM.
 *   nf [n_nodes, 128], ef [m, 128], srcs / dsts [m] (int64, node ids in [0, n_nodes)),
 *   w[3] = [384, 128], [128, 128], [128, 128]; b[3]; gamma, beta [128] (NULL: 1 and 0); fp16.
 *   out[e] = LN(ReLU(ReLU([nf[srcs[e]] | ef[e] | nf[dsts[e]]] W1 + b1) W2 + b2) W3 + b3), eps 1e-5
 *   agg (optional, fp32 [n_nodes, 128]): agg[dsts[e]] += out[e] (the fp16 values as stored),
 *   accumulated onto the caller's contents (zero it first; several edge sets may share it).
 * An index outside [0, n_nodes) reads a zero row, is left out of agg, and sets device status
 * 0x600 (gp_device_status). n_nodes <= 2^25. The [m, 384] concat never exists in memory. */
GP_API int gp_mgn_edge_update_out(int64_t m, int64_t n_nodes, const void* nf, const void* ef,
                           const int64_t* srcs, const int64_t* dsts, const void* const* w,
                           const void* const* b, const void* gamma, const void* beta, void* out,
                           float* agg, void* stream);

/* MeshGraphNet node update (graphmodel/mgn_dp.py:46-54, with the aggregates of
 * gp_mgn_edge_update_out in place of the graph's index-by-destination):
 *   out[v] = LN(MLP([nf[v] | fp16(aggs[0][v]) | ... | fp16(aggs[n_sets-1][v])])), n_sets 1 or 2,
 *   nf [n, 128], aggs[i] fp32 [n, 128], w[3] = [128 (1 + n_sets), 128], [128, 128], [128, 128].
 * The aggregates are rounded to fp16 into the per-device workspace, then read with nf through
 * two tensor maps (no concat in HBM). */
GP_API int gp_mgn_node_update_out(int64_t n, int n_sets, const void* nf, const float* const* aggs,
                           const void* const* w, const void* const* b, const void* gamma,
                           const void* beta, void* out, void* stream);

/* NeRF with view directions (apps/nerf_full/torch/model.py:5-66, use_viewdirs = True, with the
 * reference's pipelined shapes: radiance and rgb widths padded to 64). Replaces nerf_full_out
 * (apps/nerf_full/pipelined/nerf_full_pl_ext.cu:22-95). fp16.
 *   x [m, 64], d [m, 32]; w[12], b[12] = the reference's w1..w12, b1..b12:
 *   trunk w1..w8 as gp_nerf_a_out -> encoded [m, 256]
 *   out_r   [m, 64] = encoded w9 + b9                                   (w9  [256, 64])
 *   out_rgb [m, 64] = ReLU([encoded w10 + b10 | d] w11 + b11) w12 + b12 (w10 [256, 256],
 *                                                     w11 [288, 128], w12 [128, 64])
 * The ReLU after w11 follows model.py:47-50 and the reference's bulk-synchronous kernel; the
 * reference's pipelined kernel omits it. b may be NULL or hold NULL entries (no bias). Uses the
 * per-device workspace ([m, 384] fp16 plus the padded rgb weights). */
GP_API int gp_nerf_full_out(int64_t m, const void* x, const void* d, const void* const* w,
                     const void* const* b, void* out_r, void* out_rgb, void* stream);

/* GraphCast edge MLP in bf16 (as gp_gc_edges_out with dtype GP_BF16, act GP_ACT_RELU or
 * GP_ACT_SILU) for callers that cannot allocate GPU memory during a call: frameworks that own
 * every device allocation, or serving loops that must never enter an allocator. It allocates
 * nothing; the fp16 copy of the second layer's weights goes to a fixed 1 MiB buffer compiled
 * into the library (held by every GPU that loads it, until exit). The first call on a device
 * looks that buffer up (cudaGetSymbolAddress) and should come before any stream capture. Calls
 * share the buffer: calls that overlap on the GPU race and must be ordered. Its device waits use
 * the gp_set_timeout_ns budget and honour gp_set_fault_injection; a wait that runs out is
 * reported by gp_device_status like any other. It runs the single-CTA form of the kernel (the
 * regular bf16 entry point runs the CTA-pair form). No counterpart in the reference. */
GP_API int gp_gc_edges_bf16_noalloc_out(int64_t m, int act, const void* x,
                                 const void* w0, const void* b0, const void* w1, const void* b1,
                                 const void* gamma, const void* beta, void* out, void* stream);

/* gp_fused_mlp_out on HOST buffers: x_host [m, widths[0]] in, out_host [m, widths[n_layers]] out
 * (16-bit; pinned memory for overlap, pageable works but copies synchronously). The rows go in
 * chunks of chunk_rows (0: about 16 MB of rows, at least 8 chunks and 4,096 rows) through
 * double-buffered device staging: the H2D copy of chunk i+1 and the D2H copy of chunk i-1 run on two library streams while chunk
 * i computes on `stream`, so a call costs about the larger of the two PCIe directions instead of
 * their sum. Weights, biases, gamma and beta are device pointers as for gp_fused_mlp_out. Returns
 * after enqueueing; `stream` waits for the last D2H copy, so synchronising `stream` makes
 * out_host valid. No reference counterpart (the reference takes device tensors only). */
GP_API int gp_fused_mlp_host(const gp_mlp_spec* spec, int64_t m, const void* x_host,
                      const void* const* w, const void* const* b, const void* gamma,
                      const void* beta, void* out_host, int64_t chunk_rows, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Diagnostics and control (no reference counterpart: the reference has no error reporting).
 * ------------------------------------------------------------------------------------------- */
/* Message describing the last error on this thread ("" if none). */
GP_API const char* gp_last_error(void);

/* Synchronise `device` and read its status word (0 = ok, else a device-side code); with
 * clear != 0 reset it to 0. Returns GP_OK or GP_ERR_CUDA. Codes (the first one raised is kept):
 *   0x1xx-0x3xx a bounded wait ran out (producer, MMA issuer, epilogue), 0x400 weights never
 *   arrived, 0x500 dynamic shared memory misaligned, 0x600 a gather/scatter index outside
 *   [0, n_nodes) (that row read as zeros), 0x700 a wait on another tile's completion counter
 *   ran out (single-kernel wide chains), 0x800 a tile outside the chain's schedule (no memory
 *   touched). */
GP_API int gp_device_status(int device, int clear, int* status_out);

/* Budget of every device-side wait, in nanoseconds (default 2e9). 0 restores the default. */
GP_API int gp_set_timeout_ns(uint64_t ns);

/* Fault injection for tests: mode 1 makes the producer skip every input load (the single-kernel
 * wide chains: drops the completion signals between tiles) so the consumers'
 * bounded waits run out (no GPU fault; the kernel exits with a timeout status). 0 = off. */
GP_API int gp_set_fault_injection(int mode);

/* Kernel choice where several are compiled for one chain: 0 = default, 1 = the other form,
 * 2 = a third form where one exists (a chain without the requested form runs its default).
 * The MeshGraphNet family has a single-CTA and a CTA-pair kernel (the default is the faster one
 * measured for that input width). Chains with one wide first layer have a TMEM-activation kernel
 * (0), the weight-streaming kernel (1) and a CTA-pair TMEM kernel (2). BERT-large FFN and DLRM top
 * run layer by layer (0) or as one kernel with their intermediates in rings of row blocks (1).
 * Process-wide; for A/B measurement and tests. The environment variable GP_KERNEL_VARIANT sets the
 * initial value. No reference counterpart. */
GP_API int gp_set_kernel_variant(int variant);

/* Number of kernels this library has launched in this process (for launch-count claims). */
GP_API uint64_t gp_launch_count(void);

/* The launch-overlap bookkeeping of one launch on `stream`, without launching (diagnostics and
 * tests). Ranges: kinds 0 = weights / per-column parameters, 1 = input rows, 2 = written,
 * 3 = writes not listed (ptr and bytes ignored). Returns the early-read bits such a launch would
 * get (1: parameters, 2: input rows may be read before the previous kernel completes; 0 when
 * they overlap what the stream's last chain launch writes, when the stream has no record, or with
 * GP_PDL=0 / 2), or a negative GP_ERR_*; with record != 0 the ranges' writes become the stream's
 * record, as a real launch's would. No reference counterpart. */
GP_API int gp_debug_pdl_flags(void* stream, int n, const void* const* ptrs, const uint64_t* bytes,
                              const int* kinds, int record);

#ifdef __cplusplus
}
#endif

#endif /* GPIPES_H_ */
