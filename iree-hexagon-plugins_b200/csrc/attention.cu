// Fused attention dispatch (placeholder until the tcgen05 kernel lands).
#include "runtime_common.h"

extern "C" hxb_status_t hxb_attention_f16(const void* Q, const void* K, const void* V,
                                          void* O, int64_t BH, int64_t Sq, int64_t Skv,
                                          int64_t D, float scale, int causal,
                                          void* stream) {
  (void)Q; (void)K; (void)V; (void)O; (void)BH; (void)Sq; (void)Skv; (void)D;
  (void)scale; (void)causal; (void)stream;
  return hxb::fail(HXB_STATUS_UNSUPPORTED, "attention: not built yet");
}
