// Causal FlashAttention forward on tcgen05 (include/c3cu.h, c3cu_flash_attn_fwd).
// The reference has no attention kernel; this translation unit owns the fault word
// that the attention kernel reports through.
#include "common.cuh"
#include "host_util.h"

C3CU_FAULT_ACCESSORS(attn)
