// Batched decode of independent sequences (qne_batch_*): placeholder until the batched
// runner lands; every entry point reports that it is unavailable.
#include "../../include/qne.h"
#include "model.hpp"

extern "C" {
static qne_status unavailable() { return QNE_EINVAL; }
qne_status qne_batch_create(qne_model*, uint32_t, uint32_t, qne_batch** out) { if (out) *out = nullptr; return unavailable(); }
void qne_batch_free(qne_batch*) {}
qne_status qne_batch_set_page_table(qne_batch*, const uint32_t*, size_t) { return unavailable(); }
qne_status qne_batch_reset(qne_batch*) { return unavailable(); }
qne_status qne_batch_step(qne_batch*, const uint32_t*, const uint32_t*, float*, uint32_t*) { return unavailable(); }
qne_status qne_batch_decode_async(qne_batch*, uint32_t) { return unavailable(); }
qne_status qne_batch_tokens(qne_batch*, uint32_t*, uint32_t*) { return unavailable(); }
qne_status qne_batch_fill_synthetic(qne_batch*, uint32_t, uint32_t, uint32_t, uint64_t) { return unavailable(); }
qne_status qne_batch_sync(qne_batch*, uint32_t) { return unavailable(); }
size_t qne_gemm_scratch_bytes(const qne_matrix*, int) { return 0; }
qne_status qne_gemm(const qne_matrix*, const float*, int, float*, int, void*, size_t, void*) { return unavailable(); }
}
