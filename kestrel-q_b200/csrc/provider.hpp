// Device weight provider internals (shared by the GDN / QSA ABI units).
#pragma once

#include <memory>
#include <vector>

#include "kernels.hpp"
#include "kq_model.h"
#include "kq_weight_provider.h"
#include "runtime.hpp"

constexpr uint32_t kProviderMagic = 0x4b514250u;   // "KQBP"

struct ProviderTensor {
    kq_semantic_tensor desc;   // first member: handed out as the descriptor
    bool is_vector = false;
    kqb::QMatrix m{};          // matrices (device)
    float *vec_dev = nullptr;  // vectors (device copy)
    std::vector<float> vec_host;
    uint64_t bytes = 0;
    void *owned = nullptr;
    // A GDN output projection kept in the model GGUF's tiled column order:
    // column head position of every canonical value head (host and device
    // copies, width `head_width`), empty for canonical columns.
    std::vector<int32_t> col_heads;
    int32_t *col_heads_dev = nullptr;
    uint32_t head_width = 0;
    // A semantic stored as two separate tensors (the QSA index projection:
    // INDEX_QUERY then INDEX_KEY part; the routed gate/up projection: GATE
    // then UP part), each its own record.
    ProviderTensor *parts[2] = {nullptr, nullptr};
    // A routed-expert stack: `experts` matrices of `expert_rows` rows each,
    // expert-major in `m` (0 for plain matrices).
    uint32_t experts = 0;
    uint32_t expert_rows = 0;
};

// The record of `semantic`'s binding part `part_role`: the semantic itself
// for a whole tensor (part_role WHOLE), one of its parts for a split one;
// nullptr when the part does not exist.
ProviderTensor *provider_part(const kq_weight_provider *provider, const kq_semantic_tensor *semantic,
                              kq_binding_part_role part_role);

struct kq_weight_provider {
    uint32_t magic = kProviderMagic;
    int device = 0;
    std::vector<std::unique_ptr<ProviderTensor>> tensors;
    kq_weight_provider_metrics metrics{};
};

// Returns the provider record behind a descriptor, or nullptr when the
// descriptor was not created by `provider`.
ProviderTensor *provider_lookup(const kq_weight_provider *provider,
                                const kq_semantic_tensor *semantic);

// Makes the allocation-free linear's static scratch array resident on the
// current device `device` and records its device address (api_static.cu).
// Called when a provider is created, so that the array is in place before
// the host commits the rest of HBM.
namespace kqb {
kq_status static_scratch_prepare(int device, kq_diagnostic *diagnostic);
}  // namespace kqb
