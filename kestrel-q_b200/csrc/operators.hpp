// Operator entry points for the decoder-layer composition (api_layer.cpp):
// each enqueues its operator on device buffers under the caller's call (one
// error word and call id for the whole layer, so a failure anywhere rolls
// every sub-state of the layer back together).  Weights come from F32
// arrays when `wf` is given (host arrays through the context's upload
// cache), else from the provider tensors bound to the config.
#pragma once

#include "kq_gdn.h"
#include "kq_moe.h"
#include "kq_qsa.h"
#include "runtime.hpp"

namespace kqb {

kq_status gdn_layer_enqueue(DeviceContext *c, const kq_gdn_config *cfg, const kq_gdn_weights_f32 *wf,
                            kq_gdn_state *const *states, uint32_t batch, uint32_t tokens, const float *x,
                            const uint8_t *mask, float *y, ErrorWord err, kq_diagnostic *diag);
kq_status qsa_layer_enqueue(DeviceContext *c, const kq_qsa_config *cfg, const kq_qsa_weights_f32 *wf,
                            kq_qsa_state *const *states, uint32_t batch, uint32_t tokens, const float *x, float *y,
                            ErrorWord err, kq_diagnostic *diag);
kq_status moe_layer_enqueue(DeviceContext *c, const kq_moe_config *cfg, const kq_moe_weights_f32 *wf, const float *x,
                            uint64_t tokens, float *y, ErrorWord err, kq_diagnostic *diag);

// Committed state of a GDN state (its current buffer and initialised flag),
// and its restoration: the buffer a call replaced stays intact until the
// next call, so the state after the previous call can be put back.
struct GdnSnapshot {
    int cur;
    int initialized;
};
GdnSnapshot gdn_state_snapshot(const kq_gdn_state *s);
void gdn_state_restore(kq_gdn_state *s, const GdnSnapshot &snap);

// Committed length of a QSA state; truncation back to an earlier length
// (the cache is append-only, rows beyond the length are never read).
uint64_t qsa_state_committed_length(const kq_qsa_state *s);
void qsa_state_truncate(kq_qsa_state *s, uint64_t length);

}  // namespace kqb
