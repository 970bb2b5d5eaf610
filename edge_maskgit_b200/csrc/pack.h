// pack.h -- host-side block-format helpers (see pack.cpp).
#pragma once
#include <cstdint>
#include <vector>

namespace mgc {
// Q4_K device layout (see kernels.h): packed nibble bytes and compact scale bytes per row and
// 128-K chunk
constexpr int kQ4Row = 64, kQ4Scl = 16;
uint16_t f32_to_f16(float f);
float f16_to_f32(uint16_t h);
void q4k_get_scale_min(const uint8_t* s12, int j, int* sc, int* mn);
void pack_q8_0(const float* w, int64_t N, int64_t K, uint8_t* out);
void pack_q4_k(const float* w, int64_t N, int64_t K, uint8_t* out);
void dequant(int wtype, const uint8_t* w, int64_t N, int64_t K, float* out);
void repack(int wtype, const uint8_t* w, int N, int K, int Npad, std::vector<int8_t>& q, std::vector<float>& sc);
}  // namespace mgc
