// Host-side checks of the resident weight table (project-k3x_b200/csrc/
// resident.hpp), the same code the library runs over cudaMalloc'd memory,
// here over a host arena: the reference's hit / admitted / bypass rules
// (runtime/cuda/resident_weights.cu:104-166), payload and shape checks,
// capacity accounting, MXFP4 admission validation, and the stacked layout
// of expert stacks.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <set>
#include <vector>

#include "resident.hpp"

#define CHECK(cond)                                                              \
    do {                                                                         \
        if (!(cond)) {                                                           \
            std::fprintf(stderr, "check failed: %s (line %d)\n", #cond, __LINE__); \
            return 1;                                                            \
        }                                                                        \
    } while (0)

namespace {

struct Relayout {
    const void* scales;
    uint64_t rows, cols;
    void* out;
};

// malloc-backed arena that records what the table asks of the device.
class HostArena final : public k3xb::DeviceArena {
public:
    std::set<void*> live;
    std::vector<Relayout> relayouts;
    size_t uploads = 0, uploaded = 0;
    bool fail_next_allocation = false;

    int allocate(size_t bytes, void** out) override {
        if (fail_next_allocation) {
            fail_next_allocation = false;
            *out = nullptr;
            return K3XB_BACKEND_UNAVAILABLE;
        }
        *out = std::malloc(bytes ? bytes : 1);
        live.insert(*out);
        return K3XB_OK;
    }
    void release(void* p) noexcept override {
        live.erase(p);
        std::free(p);
    }
    int upload(void* dst, const void* src, size_t bytes) override {
        std::memcpy(dst, src, bytes);
        ++uploads;
        uploaded += bytes;
        return K3XB_OK;
    }
    int relayout_scales(const void* scales, uint64_t rows, uint64_t cols, void* out) override {
        relayouts.push_back({scales, rows, cols, out});
        return K3XB_OK;
    }
};

std::vector<uint8_t> bytes(size_t n, uint8_t seed) {
    std::vector<uint8_t> v(n);
    for (size_t i = 0; i < n; ++i) v[i] = static_cast<uint8_t>((seed * 131 + i * 7) % 251);   // never 0xFF
    return v;
}

int dense_rules() {
    HostArena arena;
    k3xb::ResidentTable t(&arena);
    const char* why = "";
    std::vector<float> w(6 * 8, 0.5f);
    k3xb_resident r{};
    // admitted
    CHECK(t.acquire({7, K3XB_WEIGHT_F32, 6, 8, 0}, w.data(), w.size() * 4, nullptr, 0, &r, &why) == K3XB_OK);
    CHECK(r.disposition == K3XB_RESIDENT_ADMITTED && r.primary && !r.secondary && !r.scales_tc);
    CHECK(r.uploaded_bytes == 192 && std::memcmp(r.primary, w.data(), 192) == 0);
    CHECK(t.counters().misses == 1 && t.counters().resident_bytes == 192 && t.counters().peak_resident_bytes == 192);
    // hit: same pointer, no copy
    const void* first = r.primary;
    const size_t uploads = arena.uploads;
    CHECK(t.acquire({7, K3XB_WEIGHT_F32, 6, 8, 0}, w.data(), w.size() * 4, nullptr, 0, &r, &why) == K3XB_OK);
    CHECK(r.disposition == K3XB_RESIDENT_HIT && r.primary == first && r.uploaded_bytes == 0);
    CHECK(arena.uploads == uploads && t.counters().hits == 1);
    // the same id as bf16 of the same shape is compatible (both dense): a new entry
    std::vector<uint16_t> b(6 * 8, 0x3f80);
    CHECK(t.acquire({7, K3XB_WEIGHT_BF16, 6, 8, 0}, b.data(), b.size() * 2, nullptr, 0, &r, &why) == K3XB_OK);
    CHECK(r.disposition == K3XB_RESIDENT_ADMITTED && t.counters().resident_bytes == 192 + 96);
    // the same id with another shape, or as MXFP4, is an extent error
    CHECK(t.acquire({7, K3XB_WEIGHT_F32, 8, 6, 0}, w.data(), w.size() * 4, nullptr, 0, &r, &why) ==
          K3XB_INVALID_EXTENT);
    std::vector<uint8_t> p(6 * 4), s(6);
    CHECK(t.acquire({7, K3XB_WEIGHT_MXFP4, 6, 8, 8}, p.data(), p.size(), s.data(), s.size(), &r, &why) ==
          K3XB_INVALID_EXTENT);
    // payload sizes must match the key; dense takes no group and no secondary bytes
    CHECK(t.acquire({8, K3XB_WEIGHT_F32, 6, 8, 0}, w.data(), 191, nullptr, 0, &r, &why) == K3XB_INVALID_EXTENT);
    CHECK(t.acquire({8, K3XB_WEIGHT_F32, 6, 8, 4}, w.data(), 192, nullptr, 0, &r, &why) == K3XB_INVALID_EXTENT);
    CHECK(t.acquire({8, K3XB_WEIGHT_F32, 6, 8, 0}, w.data(), 192, s.data(), 6, &r, &why) == K3XB_INVALID_EXTENT);
    CHECK(t.acquire({8, K3XB_WEIGHT_F32, 0, 8, 0}, w.data(), 0, nullptr, 0, &r, &why) == K3XB_INVALID_EXTENT);
    CHECK(t.acquire({8, 9, 6, 8, 0}, w.data(), 192, nullptr, 0, &r, &why) == K3XB_INVALID_EXTENT);
    // failed checks touched nothing
    CHECK(t.counters().misses == 2 && t.counters().hits == 1 && arena.live.size() == 2);
    t.clear();
    CHECK(arena.live.empty() && t.counters().resident_bytes == 0 && t.counters().peak_resident_bytes == 288);
    // after clear the same key is admitted again
    CHECK(t.acquire({7, K3XB_WEIGHT_F32, 6, 8, 0}, w.data(), w.size() * 4, nullptr, 0, &r, &why) == K3XB_OK);
    CHECK(r.disposition == K3XB_RESIDENT_ADMITTED);
    return 0;
}

int capacity_rules() {
    HostArena arena;
    k3xb::ResidentTable t(&arena);
    const char* why = "";
    std::vector<float> w(16, 1.0f);
    k3xb_resident r{};
    t.set_capacity(64 + 63);
    // exactly the payload fits
    CHECK(t.acquire({1, K3XB_WEIGHT_F32, 4, 4, 0}, w.data(), 64, nullptr, 0, &r, &why) == K3XB_OK);
    CHECK(r.disposition == K3XB_RESIDENT_ADMITTED);
    // the next one would pass the capacity: bypass, nothing kept
    CHECK(t.acquire({2, K3XB_WEIGHT_F32, 4, 4, 0}, w.data(), 64, nullptr, 0, &r, &why) == K3XB_OK);
    CHECK(r.disposition == K3XB_RESIDENT_BYPASS && !r.primary && !r.secondary && r.uploaded_bytes == 0);
    CHECK(t.counters().bypasses == 1 && t.counters().misses == 2 && t.counters().resident_bytes == 64);
    CHECK(arena.live.size() == 1);
    // a larger capacity admits it
    t.set_capacity(128);
    CHECK(t.acquire({2, K3XB_WEIGHT_F32, 4, 4, 0}, w.data(), 64, nullptr, 0, &r, &why) == K3XB_OK);
    CHECK(r.disposition == K3XB_RESIDENT_ADMITTED && t.counters().resident_bytes == 128);
    // an allocation failure is reported and counts nothing resident
    t.set_capacity(~0ull);
    arena.fail_next_allocation = true;
    CHECK(t.acquire({3, K3XB_WEIGHT_F32, 4, 4, 0}, w.data(), 64, nullptr, 0, &r, &why) == K3XB_BACKEND_UNAVAILABLE);
    CHECK(t.counters().resident_bytes == 128 && arena.live.size() == 2);
    return 0;
}

int mxfp4_rules() {
    HostArena arena;
    k3xb::ResidentTable t(&arena);
    const char* why = "";
    k3xb_resident r{};
    // 128 x 256, group 32: packed 16384 B, scales 1024 B, tcgen05 copy of the scales
    auto p = bytes(128 * 128, 1), s = bytes(128 * 8, 2);
    CHECK(t.acquire({11, K3XB_WEIGHT_MXFP4, 128, 256, 32}, p.data(), p.size(), s.data(), s.size(), &r, &why) ==
          K3XB_OK);
    CHECK(r.disposition == K3XB_RESIDENT_ADMITTED && r.secondary && r.scales_tc);
    CHECK(std::memcmp(r.primary, p.data(), p.size()) == 0 && std::memcmp(r.secondary, s.data(), s.size()) == 0);
    CHECK(r.uploaded_bytes == p.size() + s.size());
    CHECK(t.counters().resident_bytes == p.size() + 2 * s.size());
    CHECK(arena.relayouts.size() == 1 && arena.relayouts[0].scales == r.secondary &&
          arena.relayouts[0].rows == 128 && arena.relayouts[0].cols == 256 && arena.relayouts[0].out == r.scales_tc);
    // rows not a multiple of 128: kept without the tcgen05 copy
    auto p2 = bytes(5 * 32, 3), s2 = bytes(5 * 2, 4);
    CHECK(t.acquire({12, K3XB_WEIGHT_MXFP4, 5, 64, 32}, p2.data(), p2.size(), s2.data(), s2.size(), &r, &why) ==
          K3XB_OK);
    CHECK(r.secondary && !r.scales_tc && arena.relayouts.size() == 1);
    // group must divide cols; packed and scale sizes must match
    CHECK(t.acquire({13, K3XB_WEIGHT_MXFP4, 5, 64, 0}, p2.data(), p2.size(), s2.data(), s2.size(), &r, &why) ==
          K3XB_INVALID_EXTENT);
    CHECK(t.acquire({13, K3XB_WEIGHT_MXFP4, 5, 64, 48}, p2.data(), p2.size(), s2.data(), s2.size(), &r, &why) ==
          K3XB_INVALID_EXTENT);
    CHECK(t.acquire({13, K3XB_WEIGHT_MXFP4, 5, 64, 32}, p2.data(), p2.size(), s2.data(), 9, &r, &why) ==
          K3XB_INVALID_EXTENT);
    CHECK(t.acquire({13, K3XB_WEIGHT_MXFP4, 5, 64, 32}, p2.data(), p2.size(), nullptr, 10, &r, &why) ==
          K3XB_INVALID_EXTENT);
    // the reserved scale 0xFF fails admission
    s2[7] = 0xFF;
    CHECK(t.acquire({13, K3XB_WEIGHT_MXFP4, 5, 64, 32}, p2.data(), p2.size(), s2.data(), s2.size(), &r, &why) ==
          K3XB_INVALID_MXFP4);
    CHECK(arena.live.size() == 2);
    return 0;
}

int expert_stacks() {
    HostArena arena;
    k3xb::ResidentTable t(&arena);
    const char* why = "";
    const uint32_t E = 3, H = 256, I = 128;
    std::vector<std::vector<uint8_t>> keep;
    std::vector<k3xb_mxfp4_expert_host> host(E);
    for (uint32_t e = 0; e < E; ++e) {
        const size_t sz[6] = {size_t(I) * H / 2, size_t(I) * H / 32, size_t(I) * H / 2, size_t(I) * H / 32,
                              size_t(H) * I / 2, size_t(H) * I / 32};
        const uint8_t* ptr[6];
        for (int a = 0; a < 6; ++a) {
            keep.push_back(bytes(sz[a], static_cast<uint8_t>(10 * e + a)));
            ptr[a] = keep.back().data();
        }
        host[e] = {ptr[0], ptr[1], ptr[2], ptr[3], ptr[4], ptr[5]};
    }
    k3xb_resident_stack st{};
    CHECK(t.acquire_stack(40, E, H, I, host.data(), &st, &why) == K3XB_OK);
    CHECK(st.disposition == K3XB_RESIDENT_ADMITTED);
    // stacked layout: expert e's arrays at e * (per-expert bytes)
    for (uint32_t e = 0; e < E; ++e) {
        CHECK(std::memcmp(st.gate_packed + size_t(e) * I * H / 2, host[e].gate_packed, size_t(I) * H / 2) == 0);
        CHECK(std::memcmp(st.gate_scales + size_t(e) * I * H / 32, host[e].gate_scales, size_t(I) * H / 32) == 0);
        CHECK(std::memcmp(st.up_packed + size_t(e) * I * H / 2, host[e].up_packed, size_t(I) * H / 2) == 0);
        CHECK(std::memcmp(st.up_scales + size_t(e) * I * H / 32, host[e].up_scales, size_t(I) * H / 32) == 0);
        CHECK(std::memcmp(st.down_packed + size_t(e) * H * I / 2, host[e].down_packed, size_t(H) * I / 2) == 0);
        CHECK(std::memcmp(st.down_scales + size_t(e) * H * I / 32, host[e].down_scales, size_t(H) * I / 32) == 0);
    }
    const uint64_t copied = uint64_t(E) * (2 * (I * H / 2 + I * H / 32) + H * I / 2 + H * I / 32);
    CHECK(st.uploaded_bytes == copied);
    CHECK(t.counters().resident_bytes == copied + uint64_t(E) * (2 * I * H / 32 + H * I / 32));
    // the three tcgen05 re-layouts run over the whole stack
    CHECK(arena.relayouts.size() == 3);
    CHECK(arena.relayouts[0].scales == st.gate_scales && arena.relayouts[0].rows == uint64_t(E) * I &&
          arena.relayouts[0].cols == H && arena.relayouts[0].out == st.gate_scales_tc);
    CHECK(arena.relayouts[1].scales == st.up_scales && arena.relayouts[1].out == st.up_scales_tc);
    CHECK(arena.relayouts[2].scales == st.down_scales && arena.relayouts[2].rows == uint64_t(E) * H &&
          arena.relayouts[2].cols == I && arena.relayouts[2].out == st.down_scales_tc);
    // hit
    k3xb_resident_stack again{};
    CHECK(t.acquire_stack(40, E, H, I, host.data(), &again, &why) == K3XB_OK);
    CHECK(again.disposition == K3XB_RESIDENT_HIT && again.gate_packed == st.gate_packed && again.uploaded_bytes == 0);
    // the same stack id with another shape, or shapes the engine cannot tile
    CHECK(t.acquire_stack(40, E - 1, H, I, host.data(), &again, &why) == K3XB_INVALID_EXTENT);
    CHECK(t.acquire_stack(41, E, H, 96, host.data(), &again, &why) == K3XB_INVALID_EXTENT);
    CHECK(t.acquire_stack(41, 0, H, I, host.data(), &again, &why) == K3XB_INVALID_EXTENT);
    // a tensor id used for a plain weight cannot name a stack
    std::vector<float> w(4, 0.0f);
    k3xb_resident r{};
    CHECK(t.acquire({40, K3XB_WEIGHT_F32, 2, 2, 0}, w.data(), 16, nullptr, 0, &r, &why) == K3XB_INVALID_EXTENT);
    // 0xFF in one expert's scales fails the whole stack
    keep[2 * 6 + 5][3] = 0xFF;   // expert 2, down scales
    CHECK(t.acquire_stack(42, E, H, I, host.data(), &again, &why) == K3XB_INVALID_MXFP4);
    // bypass leaves null pointers
    t.set_capacity(t.counters().resident_bytes + 1);
    keep[2 * 6 + 5][3] = 0;
    CHECK(t.acquire_stack(43, E, H, I, host.data(), &again, &why) == K3XB_OK);
    CHECK(again.disposition == K3XB_RESIDENT_BYPASS && !again.gate_packed && !again.down_scales_tc);
    CHECK(arena.live.size() == 1);
    return 0;
}

}  // namespace

int main() {
    if (dense_rules() || capacity_rules() || mxfp4_rules() || expert_stacks()) return 1;
    std::printf("resident ok\n");
    return 0;
}
