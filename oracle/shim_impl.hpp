// ORACLE / TEST INFRASTRUCTURE — never linked into the product library.
// The CPU MetalContext's state (pass workspace, KV cache), shared by the shim's
// translation units (ref_shim.cpp: GPT members, codec_shim.cpp: codec members).
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "mit2/metal_context.hpp"

namespace mit2 {

struct MetalContext::Impl {
    std::vector<uint8_t> ws;
    size_t cursor = 0, scratch = 0;
    bool pass = false;
    std::vector<float> kv;  // [layer][K|V][capacity][width]
    uint32_t kv_layers = 0, kv_cap = 0, kv_width = 0;
    uint64_t submissions = 0;

    float* f(PassSlot s) { return reinterpret_cast<float*>(ws.data() + s.byte_offset); }
    // metal_context.mm:473-485 (256-byte aligned bump allocator)
    PassSlot alloc(uint32_t n) {
        const size_t off = cursor;
        cursor = (off + size_t(n) * 4 + 255) & ~size_t(255);
        if (cursor > ws.size())
            throw std::runtime_error("pass workspace overflow: need " + std::to_string(cursor) + " bytes, capacity " +
                                     std::to_string(ws.size()));
        return PassSlot{static_cast<uint32_t>(off), n};
    }
    float* K(uint32_t l) { return kv.data() + size_t(l) * 2 * kv_cap * kv_width; }
    float* V(uint32_t l) { return K(l) + size_t(kv_cap) * kv_width; }
    void require_pass(const char* what) {
        if (!pass) throw std::logic_error(std::string(what) + " outside pass");
    }
};

}  // namespace mit2
