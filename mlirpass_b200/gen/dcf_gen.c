/* dcf_gen.c — fast generators for the synthetic fold workloads.
 *
 * Host C, no CUDA.  Restates, element for element, the numpy definitions
 * in mlirpass_b200/workloads.py (which stay the specification) so that the
 * full-size configurations (hundreds of MB to GB of dense literals) are
 * generated in seconds:
 *   - SplitMix64 outputs start+1 .. start+n for a seed (the generator of
 *     mlirpass's fuzzer, fuzz/src/rng.rs:1-38);
 *   - uniform f32 in [lo, hi): the top 24 bits of each output as a double
 *     fraction, lo + (hi - lo) * u in double, rounded once to f32;
 *   - uniform bf16 bit patterns: the f32 above rounded to nearest even;
 *   - uppercase hex of raw bytes (the body of a dense<"0x…"> literal).
 * Built with -ffp-contract=off so that no multiply-add is fused.  Large
 * arrays are split over host threads; each element depends on its index
 * only, so the split does not change any value.
 */
#define _GNU_SOURCE
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <unistd.h>

#define GOLDEN 0x9E3779B97F4A7C15ull
#define M1 0xBF58476D1CE4E5B9ull
#define M2 0x94D049BB133111EBull

static inline uint64_t mix(uint64_t z) {
  z = (z ^ (z >> 30)) * M1;
  z = (z ^ (z >> 27)) * M2;
  return z ^ (z >> 31);
}

static inline float uniform_one(uint64_t z, double lo, double hi) {
  const double u = (double)(z >> 40) / 16777216.0;
  const double v = lo + (hi - lo) * u;
  return (float)v;
}

enum { K_SPLITMIX, K_UNIFORM_F32, K_UNIFORM_BF16, K_HEX };

typedef struct {
  int kind;
  uint64_t seed, start, lo_i, hi_i; /* element range [lo_i, hi_i) */
  double lo, hi;
  const uint8_t* in;
  void* out;
} Part;

static void run_part(const Part* p) {
  static const char digits[] = "0123456789ABCDEF";
  for (uint64_t i = p->lo_i; i < p->hi_i; i++) {
    switch (p->kind) {
      case K_SPLITMIX:
        ((uint64_t*)p->out)[i] = mix(p->seed + (p->start + i + 1) * GOLDEN);
        break;
      case K_UNIFORM_F32:
        ((float*)p->out)[i] = uniform_one(mix(p->seed + (i + 1) * GOLDEN), p->lo, p->hi);
        break;
      case K_UNIFORM_BF16: {
        union {
          float f;
          uint32_t u;
        } x;
        x.f = uniform_one(mix(p->seed + (i + 1) * GOLDEN), p->lo, p->hi);
        const uint32_t r = x.u + 0x7FFFu + ((x.u >> 16) & 1u);
        ((uint16_t*)p->out)[i] = (uint16_t)(r >> 16);
        break;
      }
      default: {
        char* o = (char*)p->out;
        o[2 * i] = digits[p->in[i] >> 4];
        o[2 * i + 1] = digits[p->in[i] & 15];
      }
    }
  }
}

static void* thread_main(void* arg) {
  run_part((const Part*)arg);
  return NULL;
}

/* Split [0, n) into one contiguous range per thread (up to 64). */
static void run(Part base, uint64_t n) {
  long cores = sysconf(_SC_NPROCESSORS_ONLN);
  int t = n < (1u << 20) ? 1 : (int)(cores < 1 ? 1 : cores > 64 ? 64 : cores);
  Part parts[64];
  pthread_t th[64];
  int started[64] = {0};
  for (int k = 0; k < t; k++) {
    parts[k] = base;
    parts[k].lo_i = n * (uint64_t)k / (uint64_t)t;
    parts[k].hi_i = n * (uint64_t)(k + 1) / (uint64_t)t;
  }
  for (int k = 1; k < t; k++) started[k] = pthread_create(&th[k], NULL, thread_main, &parts[k]) == 0;
  run_part(&parts[0]);
  for (int k = 1; k < t; k++) {
    if (started[k]) pthread_join(th[k], NULL);
    else run_part(&parts[k]);
  }
}

void dcg_splitmix64(uint64_t seed, uint64_t start, uint64_t n, uint64_t* out) {
  Part p = {K_SPLITMIX, seed, start, 0, 0, 0.0, 0.0, NULL, out};
  run(p, n);
}

void dcg_uniform_f32(uint64_t seed, uint64_t n, double lo, double hi, float* out) {
  Part p = {K_UNIFORM_F32, seed, 0, 0, 0, lo, hi, NULL, out};
  run(p, n);
}

void dcg_uniform_bf16(uint64_t seed, uint64_t n, double lo, double hi, uint16_t* out) {
  Part p = {K_UNIFORM_BF16, seed, 0, 0, 0, lo, hi, NULL, out};
  run(p, n);
}

void dcg_hex_upper(const uint8_t* in, uint64_t n, char* out) {
  Part p = {K_HEX, 0, 0, 0, 0, 0.0, 0.0, in, out};
  run(p, n);
}
