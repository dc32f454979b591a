// hex_host.cpp — decoding the hex body of a dense<"0x…"> literal on the
// host, while it is copied into a page-locked staging slot.
//
// The pass driver moves every constant it folds to the GPU.  Copying the
// literal's text and decoding it on the device sends two bytes over PCIe
// for every byte of data; decoding while staging sends one.  The copy into
// the staging slot has to touch every text byte anyway (the text lives in
// pageable memory), so the decode costs little more than the memcpy it
// replaces: 64 characters become 32 bytes per AVX-512 step (32 characters
// per AVX2 step where AVX-512 is missing), with the digit check folded in.
// Upper and lower case are accepted, as by the device decoder; anything
// else is reported as an invalid literal.
#include <immintrin.h>

#include <cstddef>
#include <cstdint>

#include "engine.h"

namespace dco {

namespace {

// 0..15 for a hex digit, 0xFF otherwise.
struct NibbleTable {
  uint8_t v[256];
  NibbleTable() {
    for (int c = 0; c < 256; c++) v[c] = 0xFF;
    for (int c = 0; c < 10; c++) v['0' + c] = (uint8_t)c;
    for (int c = 0; c < 6; c++) {
      v['A' + c] = (uint8_t)(10 + c);
      v['a' + c] = (uint8_t)(10 + c);
    }
  }
};
const NibbleTable kNib;

bool decode_scalar(const char* in, size_t nbytes, uint8_t* out) {
  uint8_t bad = 0;
  for (size_t i = 0; i < nbytes; i++) {
    const uint8_t h = kNib.v[(uint8_t)in[2 * i]], l = kNib.v[(uint8_t)in[2 * i + 1]];
    bad |= (uint8_t)((h | l) & 0xF0);
    out[i] = (uint8_t)((h << 4) | (l & 15));
  }
  return bad == 0;
}

__attribute__((target("avx2"))) bool decode_avx2(const char* in, size_t nbytes, uint8_t* out) {
  const __m256i c0 = _mm256_set1_epi8('0'), ca = _mm256_set1_epi8('a'), c20 = _mm256_set1_epi8(0x20);
  const __m256i nine = _mm256_set1_epi8(9), five = _mm256_set1_epi8(5), ten = _mm256_set1_epi8(10);
  const __m256i weights = _mm256_set1_epi16(0x0110);  // high nibble x16 + low nibble x1
  __m256i ok = _mm256_set1_epi8(-1);
  size_t i = 0;
  for (; i + 16 <= nbytes; i += 16) {
    const __m256i v = _mm256_loadu_si256((const __m256i*)(in + 2 * i));
    // digits: v - '0' in 0..9; letters: (v | 0x20) - 'a' in 0..5 (only
    // 'A'..'F' and 'a'..'f' map there)
    const __m256i d = _mm256_sub_epi8(v, c0);
    const __m256i a = _mm256_sub_epi8(_mm256_or_si256(v, c20), ca);
    const __m256i is_d = _mm256_cmpeq_epi8(_mm256_min_epu8(d, nine), d);
    const __m256i is_a = _mm256_cmpeq_epi8(_mm256_min_epu8(a, five), a);
    ok = _mm256_and_si256(ok, _mm256_or_si256(is_d, is_a));
    const __m256i nib = _mm256_blendv_epi8(_mm256_add_epi8(a, ten), d, is_d);
    const __m256i w = _mm256_maddubs_epi16(nib, weights);  // 16 words, each one byte's value
    const __m256i p = _mm256_packus_epi16(w, w);          // bytes 0-7 | 0-7 | 8-15 | 8-15 (per lane)
    const __m256i q = _mm256_permute4x64_epi64(p, 0x08);  // qwords 0 and 2 to the low half
    _mm_storeu_si128((__m128i*)(out + i), _mm256_castsi256_si128(q));
  }
  const bool all = _mm256_movemask_epi8(ok) == -1;
  return decode_scalar(in + 2 * i, nbytes - i, out + i) && all;
}

// The same steps on 64 characters at a time (AVX-512BW): the digit checks
// give lane masks, and a permutation gathers the two 128-bit lanes' packed
// bytes.
__attribute__((target("avx512bw,avx512f,avx2"))) bool decode_avx512(const char* in, size_t nbytes, uint8_t* out) {
  const __m512i c0 = _mm512_set1_epi8('0'), ca = _mm512_set1_epi8('a'), c20 = _mm512_set1_epi8(0x20);
  const __m512i nine = _mm512_set1_epi8(9), five = _mm512_set1_epi8(5), ten = _mm512_set1_epi8(10);
  const __m512i weights = _mm512_set1_epi16(0x0110);
  const __m512i order = _mm512_set_epi64(7, 5, 3, 1, 6, 4, 2, 0);
  __mmask64 ok = ~(__mmask64)0;
  size_t i = 0;
  for (; i + 32 <= nbytes; i += 32) {
    const __m512i v = _mm512_loadu_si512((const void*)(in + 2 * i));
    const __m512i d = _mm512_sub_epi8(v, c0);
    const __m512i a = _mm512_sub_epi8(_mm512_or_si512(v, c20), ca);
    const __mmask64 is_d = _mm512_cmple_epu8_mask(d, nine);
    const __mmask64 is_a = _mm512_cmple_epu8_mask(a, five);
    ok &= is_d | is_a;
    const __m512i nib = _mm512_mask_blend_epi8(is_d, _mm512_add_epi8(a, ten), d);
    const __m512i w = _mm512_maddubs_epi16(nib, weights);
    const __m512i p = _mm512_packus_epi16(w, w);           // per 128-bit lane: 8 bytes, then the same 8
    const __m512i q = _mm512_permutexvar_epi64(order, p);  // the four distinct qwords first
    _mm256_storeu_si256((__m256i*)(out + i), _mm512_castsi512_si256(q));
  }
  const bool all = ok == ~(__mmask64)0;
  return decode_avx2(in + 2 * i, nbytes - i, out + i) && all;
}

int simd_level() {
  static const int v = __builtin_cpu_supports("avx512bw") ? 2 : __builtin_cpu_supports("avx2") ? 1 : 0;
  return v;
}

}  // namespace

bool decode_hex_host(const char* in, size_t nbytes, uint8_t* out) {
  switch (simd_level()) {
    case 2: return decode_avx512(in, nbytes, out);
    case 1: return decode_avx2(in, nbytes, out);
    default: return decode_scalar(in, nbytes, out);
  }
}

}  // namespace dco
