// ref_shim.hpp — plain C views of a MoE layer and a KDA block, shared by
// the test-infrastructure shims that marshal them into the reference's C++
// API (ref_shim.cpp, ref_b200.cpp). Field order is what oracle/oracle.py
// passes over ctypes.
#pragma once

#include <cstddef>
#include <cstdint>

extern "C" {

struct k3xr_moe_layer {
    std::size_t hidden, inter, experts, top_k, shared_inter;
    const std::uint16_t* router;
    const float* correction;
    const std::uint8_t* gate_packed;
    const std::uint8_t* gate_scales;
    const std::uint8_t* up_packed;
    const std::uint8_t* up_scales;
    const std::uint8_t* down_packed;
    const std::uint8_t* down_scales;
    const std::uint16_t* shared_gate;
    const std::uint16_t* shared_up;
    const std::uint16_t* shared_down;
    int activation;  // 0 = SwiGLU (situ_glu with beta 2^64, no linear bound), 1 = SiTU
    float situ_beta, situ_linear_beta;
    std::size_t latent;                 // LatentMoE width (0: plain; k3xr_official_moe needs > 0)
    const std::uint16_t* routed_down;   // [L][H]
    const std::uint16_t* routed_norm;   // [L]
    const std::uint16_t* routed_up;     // [H][L]
    float latent_eps;
};

struct k3xr_kda_weights {
    std::size_t hidden, heads, head_dim, conv_width;
    float eps, gate_lower_bound;
    const std::uint16_t *q_proj, *k_proj, *v_proj;
    const float *q_conv, *k_conv, *v_conv;
    const std::uint16_t* f_a_proj;
    const std::uint16_t* f_b_proj;
    const float* a_log;
    const float* dt_bias;
    const std::uint16_t* b_proj;
    const std::uint16_t* g_proj;
    const float* o_norm;
    const std::uint16_t* o_proj;
};

}  // extern "C"
