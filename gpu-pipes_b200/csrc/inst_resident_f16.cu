// fp16 instantiations of the weight-resident chain kernel.
//
// Default form per input width (measured on B200, 1,048,576 rows): the CTA-pair kernel for
// K0 = 384 (half the weights per CTA leaves room for a deeper x ring), the single-CTA kernel for
// K0 <= 256. The other form of the same chain is registered as variant 1.
#include <cstring>

#include "resident_launch.cuh"

namespace gp {
// ACTS packs one activation per layer, 4 bits each, layer 0 in the low bits.
constexpr uint32_t kReluReluNone = GP_ACT_RELU | (GP_ACT_RELU << 4);

#define GP_MGN(NAME, K0, TAIL)                                                                  \
  int launch_##NAME##_pair(const LaunchCtx& c) {                                               \
    return launch_resident_pair<__half, K0, 128, 3, kReluReluNone, TAIL>(c);                   \
  }                                                                                            \
  int launch_##NAME##_single(const LaunchCtx& c) {                                             \
    return launch_resident<__half, K0, 128, 3, kReluReluNone, TAIL>(c);                        \
  }
GP_MGN(mgn_ln_f16_k384, 384, kTailLayerNorm)
GP_MGN(mgn_ln_f16_k256, 256, kTailLayerNorm)
GP_MGN(mgn_ln_f16_k128, 128, kTailLayerNorm)
GP_MGN(mgn_nl_f16_k384, 384, kTailNone)
GP_MGN(mgn_nl_f16_k256, 256, kTailNone)
GP_MGN(mgn_nl_f16_k128, 128, kTailNone)
#undef GP_MGN

// single GEMM and two-GEMM probes (known-answer tests of the tcgen05 paths), both forms
int launch_probe_1l_f16_k128_single(const LaunchCtx& c) { return launch_resident<__half, 128, 128, 1, 0u, kTailNone>(c); }
int launch_probe_2l_f16_k128_single(const LaunchCtx& c) { return launch_resident<__half, 128, 128, 2, 0u, kTailNone>(c); }
int launch_probe_1l_f16_k128_pair(const LaunchCtx& c) { return launch_resident_pair<__half, 128, 128, 1, 0u, kTailNone>(c); }
int launch_probe_2l_f16_k128_pair(const LaunchCtx& c) { return launch_resident_pair<__half, 128, 128, 2, 0u, kTailNone>(c); }
}  // namespace gp
