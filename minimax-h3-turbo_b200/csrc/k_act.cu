// Translation unit: the activation-side kernels -- rotate + quantise (rotq.cuh), RMSNorm + modulation and the gated
// residual (rmsmod.cuh), q/k norm + RoPE (rope.cuh), the attention merge (attn_merge.cuh).
#include "attn_merge.cuh"
#include "launch.h"
#include "rmsmod.cuh"
#include "rope.cuh"
#include "rotq.cuh"

namespace h3b {

H3B_DEVICE_ERROR_ACCESSOR(device_error_act)

}  // namespace h3b
