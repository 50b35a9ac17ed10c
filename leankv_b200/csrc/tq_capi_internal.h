// tq_capi_internal.h — helpers shared by the C-ABI translation units.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "leankv_tq.h"
#include "tq_attn.h"

namespace tq {

tq_status set_error(tq_status s, const char* fmt, ...);
void clear_error();   // empty the calling thread's last-error message
tq_status cuda_status(cudaError_t e, const char* what);
int log2_pow2(int64_t v);
float fwht_norm(int d);
size_t block_bytes(int type);
size_t dtype_bytes(int dt);
bool dtype_ok(int dt);
bool type_ok(int t);
// checks a decode-attention argument block and fills the kernel's run description and work plan
tq_status attn_check(const tq_decode_attention_args* a, AttnRun* r, AttnPlan* p);
// checks a paged-cache description for `batch` sequences; *shift = log2(page_size)
tq_status pages_check(const tq_kv_pages* pg, int batch, int* shift);

}  // namespace tq
