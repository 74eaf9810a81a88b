// Portable SHA-256 (FIPS 180-4), used to verify SPYR8 artifact checksums.  The
// reference computes the same digest with Windows BCrypt
// (optimized/native/src/neural/srcpyr/SrcPyrModel.cpp:87-158).
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>

namespace aeisu {

class Sha256 {
public:
    Sha256();
    void update(const uint8_t* data, size_t bytes);
    std::array<uint8_t, 32> finish();

private:
    void block(const uint8_t* p);
    uint32_t h_[8];
    uint8_t buf_[64];
    size_t fill_ = 0;
    uint64_t total_ = 0;
};

}  // namespace aeisu
