// attn_sm100.cu — flash-attention forward for B200 (sm_100a). (kernel added next)
#include "lvb_internal.h"

namespace lvb {

int attn_launch(const lvb_attn_desc* d, const void* Q, const void* K, const void* V, void* O,
                float* lse, cudaStream_t stream, DeviceState* dev) {
  return fail(LVB_ERR_UNSUPPORTED, "lvb_attention_fwd", "attention kernel not built yet");
}

}  // namespace lvb
