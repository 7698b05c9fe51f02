// fp16 instantiations of the weight-resident chain kernel.
#include <cstring>

#include "resident_launch.cuh"

namespace gp {
// ACTS packs one activation per layer, 4 bits each, layer 0 in the low bits.
constexpr uint32_t kReluReluNone = GP_ACT_RELU | (GP_ACT_RELU << 4);

int launch_mgn_ln_f16_k384(const LaunchCtx& c) { return launch_resident_pair<__half, 384, 128, 3, kReluReluNone, kTailLayerNorm>(c); }
int launch_mgn_ln_f16_k256(const LaunchCtx& c) { return launch_resident_pair<__half, 256, 128, 3, kReluReluNone, kTailLayerNorm>(c); }
int launch_mgn_ln_f16_k128(const LaunchCtx& c) { return launch_resident_pair<__half, 128, 128, 3, kReluReluNone, kTailLayerNorm>(c); }
int launch_mgn_nl_f16_k384(const LaunchCtx& c) { return launch_resident_pair<__half, 384, 128, 3, kReluReluNone, kTailNone>(c); }
int launch_mgn_nl_f16_k256(const LaunchCtx& c) { return launch_resident_pair<__half, 256, 128, 3, kReluReluNone, kTailNone>(c); }
int launch_mgn_nl_f16_k128(const LaunchCtx& c) { return launch_resident_pair<__half, 128, 128, 3, kReluReluNone, kTailNone>(c); }
int launch_probe_1l_f16_k128(const LaunchCtx& c) { return launch_resident<__half, 128, 128, 1, 0u, kTailNone>(c); }
int launch_probe_2l_f16_k128(const LaunchCtx& c) { return launch_resident<__half, 128, 128, 2, 0u, kTailNone>(c); }
// single-CTA forms of the same chains (variant 1), and pair probes
int launch_mgn_ln_f16_k384_single(const LaunchCtx& c) { return launch_resident<__half, 384, 128, 3, kReluReluNone, kTailLayerNorm>(c); }
int launch_mgn_ln_f16_k256_single(const LaunchCtx& c) { return launch_resident<__half, 256, 128, 3, kReluReluNone, kTailLayerNorm>(c); }
int launch_probe_1l_f16_k128_pair(const LaunchCtx& c) { return launch_resident_pair<__half, 128, 128, 1, 0u, kTailNone>(c); }
int launch_probe_2l_f16_k128_pair(const LaunchCtx& c) { return launch_resident_pair<__half, 128, 128, 2, 0u, kTailNone>(c); }
}  // namespace gp
