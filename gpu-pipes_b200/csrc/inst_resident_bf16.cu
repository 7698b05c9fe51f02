// bf16 instantiations of the weight-resident chain kernel (same defaults as the fp16 ones).
#include <cstring>

#include "resident_launch.cuh"

namespace gp {
constexpr uint32_t kReluReluNone = GP_ACT_RELU | (GP_ACT_RELU << 4);

int launch_mgn_ln_bf16_k384_pair(const LaunchCtx& c) { return launch_resident_pair<__nv_bfloat16, 384, 128, 3, kReluReluNone, kTailLayerNorm>(c); }
int launch_mgn_ln_bf16_k256_single(const LaunchCtx& c) { return launch_resident<__nv_bfloat16, 256, 128, 3, kReluReluNone, kTailLayerNorm>(c); }
int launch_mgn_ln_bf16_k128_single(const LaunchCtx& c) { return launch_resident<__nv_bfloat16, 128, 128, 3, kReluReluNone, kTailLayerNorm>(c); }
}  // namespace gp
