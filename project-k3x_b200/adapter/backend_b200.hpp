// backend_b200.hpp — a k3x::ComputeBackend for B200 over libk3xb.
//
// The reference's own CUDA backend refuses compute capability 10.0
// (make_cuda_backend, runtime/cuda/backend_cuda.cu:5317-5329). This backend
// is what a maintainer adds next to it (runtime/src/backend_b200.cpp, linked
// with libk3xb.so): the hot-path methods of ComputeBackend
// (runtime/include/k3x/backend.hpp:326-462) run on the B200 through the C
// ABI of k3xb.h. A call this library cannot take (a weight without a tensor
// id, which cannot stay resident, or a shape outside these kernels) returns
// backend_unavailable, as the reference's contract asks for unsupported
// shapes (backend.hpp:357-362): nothing falls back to the CPU. A failing
// call is returned as it is.
//
// On the B200:
//   mxfp4_matvec / _group, resident_mxfp4_moe_layer (weights with a tensor id)
//                                -> k3xb_acquire_weight + k3xb_mxfp4_matvec_host /
//                                   k3xb_resident_moe_layer_host (the CPU backend's products)
//   dense_matvec / _group, dense_situ_mlp (weights with a tensor id)
//                                -> k3xb_acquire_weight (f32) + k3xb_dense_matvec_host /
//                                   k3xb_dense_situ_mlp_host (bit-identical to the CPU backend)
//   mxfp4_situ_mlp_group / _batch / _grid, mxfp4_situ_moe and their
//   prefetch / _prepared forms  -> k3xb_acquire_expert_stack + k3xb_expert_grid_host
//                                  (dims not multiples of 128: single resident
//                                  MXFP4 weights on the CUDA-core engine)
//   official_mxfp4_moe_ffn (the LatentMoE FFN of one position, its route
//   given; the call official_layer_cuda makes with host route preparation)
//                                -> k3xb_acquire_weight / _expert_stack + k3xb_official_moe_ffn_host
//   prepare_official_moe_route, official_mxfp4_moe_ffn_prepared, discard_
//   official_moe_prepared (device route preparation)
//                                -> k3xb_prepare_moe_route_host, then as above
//   official_layer_front / _tail, discard_official_layer_hidden (the
//   two-layer driver's device_closure mode; the hidden rows a slot holds stay
//   in the adapter)       -> k3xb_prepare_moe_route_host + the KDA and FFN rows
//   official_kda, host-roundtrip state  -> k3xb_acquire_weight + k3xb_kda_block_host
//   official_kda, device_seed / _continue / _publish (layers 1 and 2, the
//   reference's token rules) and discard_official_kda_device_state
//                                -> k3xb_kda_block_held (the state stays on the GPU)
// Weights are uploaded once, keyed by tensor id (BackendOptions::
// cuda_resident_bytes bounds them when cuda_weights is resident).
//
// The batched verify step (k3xb_verify_step) has no ComputeBackend method:
// it replaces Engine::forward_expert_major_block as a whole and is called
// directly.
#pragma once

#include <memory>

#include "k3x/backend.hpp"
#include "k3xb.h"

namespace k3x {

// Creates a context on `device` (k3xb_create: compute capability 10.x only)
// and wraps it. Fails with the C ABI's status (backend_unavailable without a
// GPU, unsupported_architecture on other GPUs).
Result<std::unique_ptr<ComputeBackend>> make_b200_backend(const BackendOptions& options, int device = 0);

// Wraps an existing context and takes ownership of it.
std::unique_ptr<ComputeBackend> wrap_b200_context(const BackendOptions& options, k3xb_ctx* ctx);

}  // namespace k3x
