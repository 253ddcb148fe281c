// resident.hpp — bounded table of device-resident weights keyed by tensor id.
//
// Host bookkeeping only: the device side (allocation, host->device copy, the
// tcgen05 re-layout of MXFP4 scales) is a DeviceArena the caller supplies,
// so the table's rules are the same code on the GPU path (resident.cu) and
// in the CPU test (tests/cpp/resident_check.cpp).
//
// Rules follow the reference's ResidentWeightTable::acquire
// (runtime/cuda/resident_weights.cu:104-166, keys and dispositions in
// resident_weights.cuh:17-33):
//   * a payload whose byte counts do not match (rows, cols, group) and the
//     representation is INVALID_EXTENT (valid_payload, :19-38);
//   * a tensor id seen before with other rows/cols/group, or with another
//     representation (f32 and bf16 count as one dense kind), is
//     INVALID_EXTENT (compatible, :79-89);
//   * a key already held is a HIT (no copy);
//   * otherwise a MISS; when the new entry would push the resident bytes
//     past the capacity it is a BYPASS (nothing kept, null pointers);
//   * else the entry is ADMITTED: allocated, copied, counted.
// The capacity is charged the payload bytes, as there. B200 additions:
//   * MXFP4 entries whose rows and cols are multiples of 128 also hold the
//     scales in the tcgen05 block-scale layout (charged too);
//   * a MXFP4 scale byte 0xFF (the reserved E8M0 value the reference rejects
//     in ops.cpp:36-53) fails admission with INVALID_MXFP4: the reference's
//     admission-time validation mode (CudaWeightValidationMode::admission,
//     backend.hpp:24);
//   * expert stacks (E experts' gate/up/down in the contiguous
//     [E][rows][cols] layout the grouped expert GEMM reads) are entries of
//     their own kind.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <limits>
#include <map>
#include <tuple>
#include <vector>

#include "k3xb.h"

namespace k3xb {

// Device operations the table needs. Every method returns a K3XB_* status.
class DeviceArena {
public:
    virtual ~DeviceArena() = default;
    virtual int allocate(size_t bytes, void** out) = 0;
    virtual void release(void* p) noexcept = 0;
    // Copies `bytes` host bytes to device address `dst` (ordered with the
    // later `relayout_scales`).
    virtual int upload(void* dst, const void* src, size_t bytes) = 0;
    // scales [rows][cols/32] (device) -> tcgen05 layout at `out` (device).
    virtual int relayout_scales(const void* scales, uint64_t rows, uint64_t cols, void* out) = 0;
};

struct ResidentKey {
    uint64_t tensor_id;
    int32_t representation;   // K3XB_WEIGHT_*
    uint64_t rows, cols, group;
    bool operator<(const ResidentKey& o) const {
        return std::tie(tensor_id, representation, rows, cols, group) <
               std::tie(o.tensor_id, o.representation, o.rows, o.cols, o.group);
    }
};

// Byte offsets of one entry's arrays inside its single device allocation.
struct ResidentLayout {
    // K3XB_WEIGHT_F32 / BF16: part[0] = values. MXFP4: part[0] = packed,
    // part[1] = scales, part[2] = tcgen05 scales (or absent). Expert stack:
    // gate packed, gate scales, up packed, up scales, down packed, down
    // scales, then the three tcgen05 scale arrays.
    size_t offset[9] = {};
    size_t bytes[9] = {};
    int parts = 0;
    size_t total = 0;     // allocation size (parts 256-byte aligned)
    size_t counted = 0;   // bytes charged against the capacity: sum of the parts
    void add(size_t b) {
        const size_t at = (total + 255) / 256 * 256;
        offset[parts] = at;
        bytes[parts] = b;
        ++parts;
        total = at + b;
        counted += b;
    }
};

struct ResidentCounters {
    uint64_t hits = 0, misses = 0, bypasses = 0;
    uint64_t resident_bytes = 0, peak_resident_bytes = 0, uploaded_bytes = 0;
};

class ResidentTable {
public:
    explicit ResidentTable(DeviceArena* arena) : arena_(arena) {}
    ResidentTable(const ResidentTable&) = delete;
    ResidentTable& operator=(const ResidentTable&) = delete;
    ~ResidentTable() { clear(); }

    void set_capacity(uint64_t bytes) { capacity_ = bytes; }
    uint64_t capacity() const { return capacity_; }
    const ResidentCounters& counters() const { return counters_; }

    // Frees every entry (the reference's table destructor).
    void clear() {
        for (auto& [key, e] : entries_) arena_->release(e.base);
        entries_.clear();
        meta_.clear();
        counters_.resident_bytes = 0;
    }

    static bool dense(int32_t r) { return r == K3XB_WEIGHT_F32 || r == K3XB_WEIGHT_BF16; }

    // Byte counts the key implies, or false when the key is malformed
    // (valid_payload's arithmetic, with overflow guards).
    static bool payload_sizes(const ResidentKey& k, size_t* primary, size_t* secondary) {
        if (!k.rows || !k.cols || k.rows > std::numeric_limits<uint64_t>::max() / k.cols) return false;
        const uint64_t n = k.rows * k.cols;
        switch (k.representation) {
            case K3XB_WEIGHT_F32:
                if (k.group || n > std::numeric_limits<uint64_t>::max() / 4) return false;
                *primary = n * 4;
                *secondary = 0;
                return true;
            case K3XB_WEIGHT_BF16:
                if (k.group || n > std::numeric_limits<uint64_t>::max() / 2) return false;
                *primary = n * 2;
                *secondary = 0;
                return true;
            case K3XB_WEIGHT_MXFP4:
                if (!k.group || k.cols % k.group || k.cols % 2) return false;
                *primary = n / 2;
                *secondary = n / k.group;
                return true;
            default:
                return false;
        }
    }

    static bool tc_layout(const ResidentKey& k) {
        return k.representation == K3XB_WEIGHT_MXFP4 && k.group == 32 && k.rows % 128 == 0 &&
               k.cols % 128 == 0;
    }

    static ResidentLayout layout_of(const ResidentKey& k) {
        ResidentLayout l;
        size_t p = 0, s = 0;
        if (k.representation == K3XB_WEIGHT_EXPERT_STACK) {
            // rows = experts, cols = hidden, group = inter
            const size_t E = k.rows, H = k.cols, I = k.group;
            for (int m = 0; m < 2; ++m) {   // gate, up: [E][I][H]
                l.add(E * I * (H / 2));
                l.add(E * I * (H / 32));
            }
            l.add(E * H * (I / 2));         // down: [E][H][I]
            l.add(E * H * (I / 32));
            l.add(E * I * (H / 32));
            l.add(E * I * (H / 32));
            l.add(E * H * (I / 32));
            return l;
        }
        payload_sizes(k, &p, &s);
        l.add(p);
        if (s) l.add(s);
        if (tc_layout(k)) l.add(s);
        return l;
    }

    // One weight (k3xb_acquire_weight).
    int acquire(const ResidentKey& k, const void* primary, size_t primary_bytes, const void* secondary,
                size_t secondary_bytes, k3xb_resident* out, const char** why) {
        size_t p = 0, s = 0;
        if (k.representation == K3XB_WEIGHT_EXPERT_STACK || !payload_sizes(k, &p, &s) ||
            primary_bytes != p || secondary_bytes != s || !primary || (s && !secondary) ||
            !compatible(k)) {
            *why = "resident weight: payload does not match its key, or the tensor id was seen with another shape";
            return K3XB_INVALID_EXTENT;
        }
        *out = k3xb_resident{};
        if (auto it = entries_.find(k); it != entries_.end()) {
            ++counters_.hits;
            fill(it->second, out, K3XB_RESIDENT_HIT, 0);
            return K3XB_OK;
        }
        ++counters_.misses;
        if (k.representation == K3XB_WEIGHT_MXFP4 && std::memchr(secondary, 0xFF, s)) {
            *why = "resident weight: MXFP4 scale 0xFF is reserved";
            return K3XB_INVALID_MXFP4;
        }
        const ResidentLayout l = layout_of(k);
        if (!fits(l.counted)) {
            ++counters_.bypasses;
            out->disposition = K3XB_RESIDENT_BYPASS;
            return K3XB_OK;
        }
        Entry e{nullptr, l};
        int st = arena_->allocate(l.total, &e.base);
        if (st) {
            *why = "resident weight: device allocation failed";
            return st;
        }
        char* b = static_cast<char*>(e.base);
        if ((st = arena_->upload(b + l.offset[0], primary, p)) ||
            (s && (st = arena_->upload(b + l.offset[1], secondary, s))) ||
            (tc_layout(k) && (st = arena_->relayout_scales(b + l.offset[1], k.rows, k.cols, b + l.offset[2])))) {
            arena_->release(e.base);
            *why = "resident weight: upload failed";
            return st;
        }
        admit(k, e, p + s);
        fill(e, out, K3XB_RESIDENT_ADMITTED, p + s);
        return K3XB_OK;
    }

    // E experts into one stack (k3xb_acquire_expert_stack). The per-expert
    // views must stay valid for the call only.
    int acquire_stack(uint64_t stack_id, uint32_t E, uint32_t H, uint32_t I, const k3xb_mxfp4_expert_host* host,
                      k3xb_resident_stack* out, const char** why) {
        const ResidentKey k{stack_id, K3XB_WEIGHT_EXPERT_STACK, E, H, I};
        if (!E || !H || !I || H % 128 || I % 128 || !host || !compatible(k)) {
            *why = "expert stack: experts > 0, hidden and inter multiples of 128, and a stack id of this shape";
            return K3XB_INVALID_EXTENT;
        }
        for (uint32_t e = 0; e < E; ++e) {
            const k3xb_mxfp4_expert_host& x = host[e];
            if (!x.gate_packed || !x.gate_scales || !x.up_packed || !x.up_scales || !x.down_packed ||
                !x.down_scales) {
                *why = "expert stack: null expert view";
                return K3XB_INVALID_EXTENT;
            }
        }
        *out = k3xb_resident_stack{};
        if (auto it = entries_.find(k); it != entries_.end()) {
            ++counters_.hits;
            fill_stack(it->second, out, K3XB_RESIDENT_HIT, 0);
            return K3XB_OK;
        }
        ++counters_.misses;
        const size_t gp = size_t(I) * (H / 2), gs = size_t(I) * (H / 32);
        const size_t dp = size_t(H) * (I / 2), ds = size_t(H) * (I / 32);
        for (uint32_t e = 0; e < E; ++e) {
            const k3xb_mxfp4_expert_host& x = host[e];
            if (std::memchr(x.gate_scales, 0xFF, gs) || std::memchr(x.up_scales, 0xFF, gs) ||
                std::memchr(x.down_scales, 0xFF, ds)) {
                *why = "expert stack: MXFP4 scale 0xFF is reserved";
                return K3XB_INVALID_MXFP4;
            }
        }
        const ResidentLayout l = layout_of(k);
        if (!fits(l.counted)) {
            ++counters_.bypasses;
            out->disposition = K3XB_RESIDENT_BYPASS;
            return K3XB_OK;
        }
        Entry en{nullptr, l};
        int st = arena_->allocate(l.total, &en.base);
        if (st) {
            *why = "expert stack: device allocation failed";
            return st;
        }
        char* b = static_cast<char*>(en.base);
        const size_t per[6] = {gp, gs, gp, gs, dp, ds};
        for (uint32_t e = 0; e < E && !st; ++e) {
            const k3xb_mxfp4_expert_host& x = host[e];
            const void* src[6] = {x.gate_packed, x.gate_scales, x.up_packed, x.up_scales, x.down_packed,
                                  x.down_scales};
            for (int a = 0; a < 6 && !st; ++a) st = arena_->upload(b + l.offset[a] + e * per[a], src[a], per[a]);
        }
        if (!st) st = arena_->relayout_scales(b + l.offset[1], uint64_t(E) * I, H, b + l.offset[6]);
        if (!st) st = arena_->relayout_scales(b + l.offset[3], uint64_t(E) * I, H, b + l.offset[7]);
        if (!st) st = arena_->relayout_scales(b + l.offset[5], uint64_t(E) * H, I, b + l.offset[8]);
        if (st) {
            arena_->release(en.base);
            *why = "expert stack: upload failed";
            return st;
        }
        const uint64_t copied = uint64_t(E) * (2 * gp + 2 * gs + dp + ds);
        admit(k, en, copied);
        fill_stack(en, out, K3XB_RESIDENT_ADMITTED, copied);
        return K3XB_OK;
    }

private:
    struct Entry {
        void* base;
        ResidentLayout layout;
    };
    struct Meta {
        int32_t representation;
        uint64_t rows, cols, group;
    };

    bool compatible(const ResidentKey& k) const {
        auto it = meta_.find(k.tensor_id);
        if (it == meta_.end()) return true;
        const Meta& m = it->second;
        if (m.rows != k.rows || m.cols != k.cols || m.group != k.group) return false;
        return m.representation == k.representation || (dense(m.representation) && dense(k.representation));
    }

    bool fits(size_t required) const {
        return required <= capacity_ && counters_.resident_bytes <= capacity_ - required;
    }

    void admit(const ResidentKey& k, const Entry& e, uint64_t copied) {
        counters_.resident_bytes += e.layout.counted;
        if (counters_.resident_bytes > counters_.peak_resident_bytes)
            counters_.peak_resident_bytes = counters_.resident_bytes;
        counters_.uploaded_bytes += copied;
        meta_.try_emplace(k.tensor_id, Meta{k.representation, k.rows, k.cols, k.group});
        entries_.emplace(k, e);
    }

    static void fill(const Entry& e, k3xb_resident* out, int32_t disposition, uint64_t copied) {
        const char* b = static_cast<const char*>(e.base);
        out->disposition = disposition;
        out->primary = b + e.layout.offset[0];
        out->secondary = e.layout.parts > 1 ? b + e.layout.offset[1] : nullptr;
        out->scales_tc = e.layout.parts > 2 ? b + e.layout.offset[2] : nullptr;
        out->uploaded_bytes = copied;
    }

    static void fill_stack(const Entry& e, k3xb_resident_stack* out, int32_t disposition, uint64_t copied) {
        const auto at = [&](int i) { return static_cast<const uint8_t*>(e.base) + e.layout.offset[i]; };
        out->disposition = disposition;
        out->gate_packed = at(0);
        out->gate_scales = at(1);
        out->up_packed = at(2);
        out->up_scales = at(3);
        out->down_packed = at(4);
        out->down_scales = at(5);
        out->gate_scales_tc = at(6);
        out->up_scales_tc = at(7);
        out->down_scales_tc = at(8);
        out->uploaded_bytes = copied;
    }

    DeviceArena* arena_;
    uint64_t capacity_ = std::numeric_limits<uint64_t>::max();
    ResidentCounters counters_;
    std::map<ResidentKey, Entry> entries_;
    std::map<uint64_t, Meta> meta_;
};

}  // namespace k3xb
