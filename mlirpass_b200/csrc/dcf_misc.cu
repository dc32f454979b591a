// dcf_misc.cu — dispatch, grid sizing, and the data-movement kernels:
// transpose / permute (the layerwise transpose fold), the dense hex codec
// (dense<"0x…"> bodies), and the splat test.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <string>
#include <unordered_map>

#include "dcf_kernels.cuh"

namespace dcf {

size_t dtype_size(int dtype) {
  switch (dtype) {
    case DCF_I1: case DCF_I8: case DCF_F8E5M2: case DCF_F8E4M3: case DCF_F8E3M4: return 1;
    case DCF_I16: case DCF_F16: case DCF_BF16: return 2;
    case DCF_I32: case DCF_F32: return 4;
    case DCF_I64: case DCF_F64: return 8;
    default: return 0;
  }
}

static std::atomic<uint64_t> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
uint64_t launches() { return g_launches.load(std::memory_order_relaxed); }

bool is_float(int dtype) { return dtype >= DCF_F16 && dtype <= DCF_F8E3M4; }
bool is_int(int dtype) { return dtype >= DCF_I1 && dtype <= DCF_I64; }

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("DCF_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Grid = min(blocks the work needs, blocks resident on all SMs at once).
int grid_for(uint64_t work_items, const void* kernel) {
  static std::mutex mu;
  static std::unordered_map<const void*, int> occ[64];
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 63;
  int per_sm;
  {
    std::lock_guard<std::mutex> g(mu);
    if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    auto it = occ[dev].find(kernel);
    if (it == occ[dev].end()) {
      int b = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, kThreads, 0) != cudaSuccess || b < 1) b = 1;
      it = occ[dev].emplace(kernel, b).first;
    }
    per_sm = it->second;
  }
  const uint64_t resident = (uint64_t)sms[dev] * (uint64_t)per_sm;
  uint64_t need = (work_items + (uint64_t)kThreads * kUnroll - 1) / ((uint64_t)kThreads * kUnroll);
  if (need < 1) need = 1;
  return (int)(need < resident ? need : resident);
}

// The bulk-copy pipeline pays a fixed cost per CTA (barrier set-up, the
// first copies' latency, a partial last round); below this many 16 KB tiles
// per SM the plain-load kernel is used.  DCF_TMA_TILES_PER_SM overrides it.
int tma_min_tiles_per_sm() {
  static const int v = [] {
    const char* e = getenv("DCF_TMA_TILES_PER_SM");
    const int x = e ? atoi(e) : 0;
    return x > 0 ? x : 2;
  }();
  return v;
}

// Which 2-byte transpose the status-reporting entry points use: the
// bulk-tensor pipeline (DCF_TRANSPOSE=tma) or the plain-load kernel with a
// register prefetch of the next tile (the default: faster on B200).
bool transpose_tma_enabled() {
  static const bool v = [] {
    const char* e = getenv("DCF_TRANSPOSE");
    return e && std::string(e) == "tma";
  }();
  return v;
}

int sm_count_current() {
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 63;
  if (!sms[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    sms[dev] = n > 0 ? n : 1;
  }
  return sms[dev];
}

// Raise a kernel's dynamic shared memory limit once per device.
bool prepare_smem(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::unordered_map<const void*, int> done[64];
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 63;
  std::lock_guard<std::mutex> g(mu);
  auto it = done[dev].find(kernel);
  if (it != done[dev].end() && it->second >= bytes) return true;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
  // These kernels use no L1-resident data worth keeping: give shared memory
  // the whole carve-out, so that the pipelines' stages of several CTAs fit.
  cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  cudaGetLastError();
  done[dev][kernel] = bytes;
  return true;
}

int resident_per_sm(const void* kernel, int smem, int cap) {
  static std::mutex mu;
  static std::unordered_map<const void*, std::pair<int, int>> memo[64];
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 63;
  std::lock_guard<std::mutex> g(mu);
  auto it = memo[dev].find(kernel);
  if (it != memo[dev].end() && it->second.first == smem) return it->second.second < cap ? it->second.second : cap;
  int b = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, kThreads, (size_t)smem) != cudaSuccess || b < 1) {
    cudaGetLastError();
    b = 1;
  }
  memo[dev][kernel] = {smem, b};
  return b < cap ? b : cap;
}

int launch_ew(const EwLaunch& a) {
  if (op_float_binary(a.op)) return launch_float_binary(a);
  if (op_int_binary(a.op)) return launch_int_binary(a);
  if (op_convert(a.op)) return launch_convert(a);
  if (a.op == DCF_RECIPROCAL) return launch_reciprocal(a);
  return DCF_EUNSUPPORTED;
}

// ------------------------------------------------------------ transpose

// 2-byte elements, rows and cols multiples of 64: each 64x64 tile is read
// as 32-bit column pairs of two adjacent rows, 2x2-transposed in registers,
// and written to an XOR-swizzled 64x32-word shared tile, so that both the
// global reads and the global writes are 128-byte coalesced rows and the
// shared-memory accesses are free of bank conflicts.  The next tile's loads
// are issued before this tile's stores, so they are in flight meanwhile.
__device__ __forceinline__ void load_tile_b16(const uint32_t* __restrict__ in, uint64_t t, uint64_t tiles_c,
                                              uint64_t in_words, int warp, int lane, uint32_t (&a)[4],
                                              uint32_t (&b)[4]) {
  const uint64_t r0 = (t / tiles_c) * 64, c0 = (t % tiles_c) * 64;
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const int y = warp + 8 * k;
    const uint64_t row = r0 + 2 * y;
    a[k] = __ldg(in + row * in_words + c0 / 2 + lane);
    b[k] = __ldg(in + (row + 1) * in_words + c0 / 2 + lane);
  }
}

__global__ void __launch_bounds__(256) transpose_b16_kernel(const uint32_t* __restrict__ in,
                                                            uint32_t* __restrict__ out, uint64_t rows,
                                                            uint64_t cols) {
  __shared__ uint32_t s[64][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint64_t tiles_c = cols / 64, ntiles = (rows / 64) * tiles_c;
  const uint64_t in_words = cols / 2, out_words = rows / 2;
  uint32_t a[4] = {0, 0, 0, 0}, b[4] = {0, 0, 0, 0};
  if (blockIdx.x < ntiles) load_tile_b16(in, blockIdx.x, tiles_c, in_words, warp, lane, a, b);
  for (uint64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const uint64_t r0 = (t / tiles_c) * 64, c0 = (t % tiles_c) * 64;
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int y = warp + 8 * k;
      const uint32_t w0 = (a[k] & 0xFFFFu) | (b[k] << 16);
      const uint32_t w1 = (a[k] >> 16) | (b[k] & 0xFFFF0000u);
      s[2 * lane][y ^ lane] = w0;
      s[2 * lane + 1][y ^ lane] = w1;
    }
    const uint64_t tn = t + gridDim.x;
    if (tn < ntiles) load_tile_b16(in, tn, tiles_c, in_words, warp, lane, a, b);
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int R = warp + 8 * k;
      out[(c0 + R) * out_words + r0 / 2 + lane] = s[R][lane ^ (R >> 1)];
    }
    __syncthreads();
  }
}

// Any element size and shape: classic 32x32 tile with a padded column.
template <typename T>
__global__ void __launch_bounds__(256) transpose_any_kernel(const T* __restrict__ in, T* __restrict__ out,
                                                            uint64_t rows, uint64_t cols) {
  __shared__ T tile[32][33];
  const uint64_t tiles_c = (cols + 31) / 32, ntiles = ((rows + 31) / 32) * tiles_c;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (uint64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const uint64_t r0 = (t / tiles_c) * 32, c0 = (t % tiles_c) * 32;
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const uint64_t r = r0 + ty + 8 * k, c = c0 + tx;
      if (r < rows && c < cols) tile[ty + 8 * k][tx] = in[r * cols + c];
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const uint64_t oc = c0 + ty + 8 * k, orr = r0 + tx;  // out row = input col
      if (oc < cols && orr < rows) out[oc * rows + orr] = tile[tx][ty + 8 * k];
    }
    __syncthreads();
  }
}

static int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 1;
}

int launch_transpose2d(size_t es, uint64_t rows, uint64_t cols, const void* in, void* out, cudaStream_t st,
                       dcf_status* status) {
  if (rows == 0 || cols == 0) return DCF_OK;
  if (es == 2 && status && transpose_tma_enabled()) {
    const int rc = launch_transpose2_tma(in, out, rows, cols, status, st);
    if (rc != DCF_EUNSUPPORTED) return rc;
  }
  const int sms = sm_count();
  if (es == 2 && rows % 64 == 0 && cols % 64 == 0 && ((uintptr_t)in & 3) == 0 && ((uintptr_t)out & 3) == 0) {
    // one wave of persistent CTAs (as many as are resident at once)
    const uint64_t nt = (rows / 64) * (cols / 64);
    const int g = grid_for(nt * (uint64_t)kThreads * kUnroll, (const void*)transpose_b16_kernel);
    note_launch();
    transpose_b16_kernel<<<(unsigned)g, 256, 0, st>>>((const uint32_t*)in, (uint32_t*)out, rows, cols);
  } else {
    const uint64_t nt = ((rows + 31) / 32) * ((cols + 31) / 32);
    const unsigned g = (unsigned)(nt < (uint64_t)sms * 8 ? nt : (uint64_t)sms * 8);
    note_launch();
    switch (es) {
      case 1: transpose_any_kernel<uint8_t><<<g, 256, 0, st>>>((const uint8_t*)in, (uint8_t*)out, rows, cols); break;
      case 2: transpose_any_kernel<uint16_t><<<g, 256, 0, st>>>((const uint16_t*)in, (uint16_t*)out, rows, cols); break;
      case 4: transpose_any_kernel<uint32_t><<<g, 256, 0, st>>>((const uint32_t*)in, (uint32_t*)out, rows, cols); break;
      case 8: transpose_any_kernel<uint64_t><<<g, 256, 0, st>>>((const uint64_t*)in, (uint64_t*)out, rows, cols); break;
      default: return DCF_EINVAL;
    }
  }
  return cudaPeekAtLastError() == cudaSuccess ? DCF_OK : DCF_ECUDA;
}

struct PermDesc {
  int rank;
  int64_t out_shape[8];
  int64_t src_stride[8];  // input stride of the dim that output dim i reads
};

template <typename T>
__global__ void __launch_bounds__(256) permute_kernel(const T* __restrict__ in, T* __restrict__ out, uint64_t total,
                                                      PermDesc d) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t o = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total; o += stride) {
    uint64_t rem = o, off = 0;
    for (int i = d.rank - 1; i >= 0; i--) {
      const uint64_t dim = (uint64_t)d.out_shape[i];
      off += (rem % dim) * (uint64_t)d.src_stride[i];
      rem /= dim;
    }
    out[o] = in[off];
  }
}

int launch_permute(size_t es, int rank, const int64_t* in_shape, const int64_t* perms, const void* in, void* out,
                   cudaStream_t st, dcf_status* status) {
  if (rank < 1 || rank > 8) return DCF_EINVAL;
  // A swap of two contiguous groups of dims is a 2-D transpose.
  for (int split = 1; split < rank; split++) {
    bool swap = true;
    for (int i = 0; i < rank && swap; i++)
      swap = perms[i] == ((i < rank - split) ? split + i : i - (rank - split));
    if (swap) {
      uint64_t rows = 1, cols = 1;
      for (int i = 0; i < split; i++) rows *= (uint64_t)in_shape[i];
      for (int i = split; i < rank; i++) cols *= (uint64_t)in_shape[i];
      return launch_transpose2d(es, rows, cols, in, out, st, status);
    }
  }
  PermDesc d{};
  d.rank = rank;
  int64_t in_stride[8], total = 1;
  for (int i = rank - 1; i >= 0; i--) {
    if (in_shape[i] < 0) return DCF_EINVAL;
    in_stride[i] = total;
    total *= in_shape[i];
  }
  for (int i = 0; i < rank; i++) {
    if (perms[i] < 0 || perms[i] >= rank) return DCF_EINVAL;
    d.out_shape[i] = in_shape[perms[i]];
    d.src_stride[i] = in_stride[perms[i]];
  }
  if (total == 0) return DCF_OK;
  const int sms = sm_count();
  const uint64_t need = ((uint64_t)total + 255) / 256;
  const unsigned g = (unsigned)(need < (uint64_t)sms * 8 ? need : (uint64_t)sms * 8);
  note_launch();
  switch (es) {
    case 1: permute_kernel<uint8_t><<<g, 256, 0, st>>>((const uint8_t*)in, (uint8_t*)out, total, d); break;
    case 2: permute_kernel<uint16_t><<<g, 256, 0, st>>>((const uint16_t*)in, (uint16_t*)out, total, d); break;
    case 4: permute_kernel<uint32_t><<<g, 256, 0, st>>>((const uint32_t*)in, (uint32_t*)out, total, d); break;
    case 8: permute_kernel<uint64_t><<<g, 256, 0, st>>>((const uint64_t*)in, (uint64_t*)out, total, d); break;
    default: return DCF_EINVAL;
  }
  return cudaPeekAtLastError() == cudaSuccess ? DCF_OK : DCF_ECUDA;
}

// ------------------------------------------------------------ hex codec

__device__ __forceinline__ uint32_t hex2(uint32_t byte) {
  const uint32_t hi = byte >> 4, lo = byte & 15;
  const uint32_t ch = hi + 48 + (hi > 9 ? 7 : 0), cl = lo + 48 + (lo > 9 ? 7 : 0);
  return ch | (cl << 8);
}

// 8 input bytes -> 16 characters per thread (vector path when aligned).
__global__ void __launch_bounds__(256) hex_encode_kernel(const uint8_t* __restrict__ in, uint64_t nbytes,
                                                         char* __restrict__ out, int vec) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const uint64_t nv = vec ? nbytes / 8 : 0;
  for (uint64_t v = tid; v < nv; v += stride) {
    const uint2 x = __ldg((const uint2*)(in + v * 8));
    uint4 y;
    y.x = hex2(x.x & 0xFF) | (hex2((x.x >> 8) & 0xFF) << 16);
    y.y = hex2((x.x >> 16) & 0xFF) | (hex2(x.x >> 24) << 16);
    y.z = hex2(x.y & 0xFF) | (hex2((x.y >> 8) & 0xFF) << 16);
    y.w = hex2((x.y >> 16) & 0xFF) | (hex2(x.y >> 24) << 16);
    *(uint4*)(out + v * 16) = y;
  }
  for (uint64_t i = nv * 8 + tid; i < nbytes; i += stride) {
    const uint32_t h = hex2(in[i]);
    out[2 * i] = (char)(h & 0xFF);
    out[2 * i + 1] = (char)(h >> 8);
  }
}

__device__ __forceinline__ int unhex(uint32_t c) {
  if (c >= '0' && c <= '9') return (int)(c - '0');
  if (c >= 'A' && c <= 'F') return (int)(c - 'A' + 10);
  if (c >= 'a' && c <= 'f') return (int)(c - 'a' + 10);
  return -1;
}

// Decode nbytes bytes from 2*nbytes characters, threads tid, tid+stride,
// ...: 16 characters -> 8 bytes per step when the text is 16-byte aligned
// (vec).  Returns the lowest invalid character index this thread saw.
__device__ __forceinline__ uint64_t decode_span(const char* __restrict__ in, uint64_t nbytes,
                                                uint8_t* __restrict__ out, uint64_t tid, uint64_t stride, bool vec) {
  const uint64_t nv = vec ? nbytes / 8 : 0;
  uint64_t bad = ~0ull;
  for (uint64_t v = tid; v < nv; v += stride) {
    const uint4 x = __ldg((const uint4*)(in + v * 16));
    const uint32_t w[4] = {x.x, x.y, x.z, x.w};
    uint32_t o[2] = {0, 0};
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const uint32_t word = w[k / 2];
      const uint32_t c0 = (word >> ((k & 1) * 16)) & 0xFF, c1 = (word >> ((k & 1) * 16 + 8)) & 0xFF;
      const int h = unhex(c0), l = unhex(c1);
      if (h < 0 || l < 0) {
        const uint64_t at = v * 16 + 2 * k + (h < 0 ? 0 : 1);
        bad = at < bad ? at : bad;
      }
      o[k / 4] |= (uint32_t)((h << 4 | l) & 0xFF) << ((k & 3) * 8);
    }
    *(uint2*)(out + v * 8) = make_uint2(o[0], o[1]);
  }
  for (uint64_t i = nv * 8 + tid; i < nbytes; i += stride) {
    const int h = unhex((uint8_t)in[2 * i]), l = unhex((uint8_t)in[2 * i + 1]);
    if (h < 0 || l < 0) {
      const uint64_t at = 2 * i + (h < 0 ? 0 : 1);
      bad = at < bad ? at : bad;
    }
    out[i] = (uint8_t)((h << 4 | l) & 0xFF);
  }
  return bad;
}

// An invalid character records its index as the status's first_fail.
__global__ void __launch_bounds__(256) hex_decode_kernel(const char* __restrict__ in, uint64_t nbytes,
                                                         uint8_t* __restrict__ out, dcf_status* st, int vec) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  report(st, decode_span(in, nbytes, out, tid, stride, vec != 0), false);
}

// 16 characters (as four words) -> 8 bytes; `bad` gets the lowest invalid
// character index, counting from `at`.
__device__ __forceinline__ uint2 decode16(const uint32_t (&w)[4], uint64_t at, uint64_t& bad) {
  uint32_t o[2] = {0, 0};
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const uint32_t word = w[k / 2];
    const uint32_t c0 = (word >> ((k & 1) * 16)) & 0xFF, c1 = (word >> ((k & 1) * 16 + 8)) & 0xFF;
    const int h = unhex(c0), l = unhex(c1);
    if (h < 0 || l < 0) {
      const uint64_t x = at + 2 * k + (h < 0 ? 0 : 1);
      bad = x < bad ? x : bad;
    }
    o[k / 4] |= (uint32_t)((h << 4 | l) & 0xFF) << ((k & 3) * 8);
  }
  return make_uint2(o[0], o[1]);
}

// Text at any alignment m = in % 16: each lane loads the aligned 16-byte
// block under its 16 characters, takes the next block from its neighbour
// lane (the last lane loads it), and funnel-shifts the pair by m bytes.
// Reads up to 15 bytes before the text and 16 bytes after its end.  The
// loop runs whole warps (stride is a multiple of 32).
__device__ __forceinline__ uint64_t decode_span_shifted(const char* __restrict__ in, uint64_t nbytes,
                                                        uint8_t* __restrict__ out, uint64_t tid, uint64_t stride) {
  const unsigned full = 0xFFFFFFFFu;
  const int lane = threadIdx.x & 31;
  const uint32_t m = (uint32_t)((uintptr_t)in & 15);
  const uint4* base = (const uint4*)(in - m);
  const uint64_t nv = nbytes / 8;
  uint64_t bad = ~0ull;
  for (uint64_t vb = tid - lane; vb < nv; vb += stride) {
    const uint64_t v = vb + lane;
    const uint4 cur = v < nv ? __ldg(base + v) : make_uint4(0, 0, 0, 0);
    uint4 nxt;
    nxt.x = __shfl_down_sync(full, cur.x, 1);
    nxt.y = __shfl_down_sync(full, cur.y, 1);
    nxt.z = __shfl_down_sync(full, cur.z, 1);
    nxt.w = __shfl_down_sync(full, cur.w, 1);
    if (lane == 31 || v + 1 >= nv) {
      if (v < nv) nxt = __ldg(base + v + 1);
    }
    if (v < nv) {
      const uint32_t w8[8] = {cur.x, cur.y, cur.z, cur.w, nxt.x, nxt.y, nxt.z, nxt.w};
      const uint32_t sh = 8 * (m & 3);
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; k++) {
        uint32_t lo, hi;
        switch (m >> 2) {  // whole words to skip
          case 0: lo = w8[k]; hi = w8[k + 1]; break;
          case 1: lo = w8[k + 1]; hi = w8[k + 2]; break;
          case 2: lo = w8[k + 2]; hi = w8[k + 3]; break;
          default: lo = w8[k + 3]; hi = w8[k + 4]; break;
        }
        w[k] = __funnelshift_r(lo, hi, sh);
      }
      *(uint2*)(out + v * 8) = decode16(w, v * 16, bad);
    }
  }
  for (uint64_t i = nv * 8 + tid; i < nbytes; i += stride) {
    const int h = unhex((uint8_t)in[2 * i]), l = unhex((uint8_t)in[2 * i + 1]);
    if (h < 0 || l < 0) {
      const uint64_t at = 2 * i + (h < 0 ? 0 : 1);
      bad = at < bad ? at : bad;
    }
    out[i] = (uint8_t)((h << 4 | l) & 0xFF);
  }
  return bad;
}

// Many literals in one launch: blockIdx.y picks the piece, the blocks along
// x stride over it.  An invalid character anywhere sets first_fail to the
// lowest index within its piece.
__global__ void __launch_bounds__(256) hex_decode_pieces_kernel(const dcf_hex_piece* __restrict__ pieces,
                                                                dcf_status* st) {
  const dcf_hex_piece pc = pieces[blockIdx.y];
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  uint64_t bad = 0;
  if (!(pc.nchars & 1)) {
    if ((uintptr_t)pc.out & 7)
      bad = decode_span(pc.in, pc.nchars / 2, (uint8_t*)pc.out, tid, stride, false);
    else if ((uintptr_t)pc.in & 15)
      bad = decode_span_shifted(pc.in, pc.nchars / 2, (uint8_t*)pc.out, tid, stride);
    else
      bad = decode_span(pc.in, pc.nchars / 2, (uint8_t*)pc.out, tid, stride, true);
  }
  report(st, bad, false);
}

int launch_hex_encode(const void* in, uint64_t nbytes, char* out, cudaStream_t st) {
  if (nbytes == 0) return DCF_OK;
  const int vec = (((uintptr_t)in & 7) == 0 && ((uintptr_t)out & 15) == 0);
  const uint64_t need = (nbytes / 8 + 255) / 256 + 1;
  const int sms = sm_count();
  const unsigned g = (unsigned)(need < (uint64_t)sms * 8 ? need : (uint64_t)sms * 8);
  note_launch();
  hex_encode_kernel<<<g, 256, 0, st>>>((const uint8_t*)in, nbytes, out, vec);
  return cudaPeekAtLastError() == cudaSuccess ? DCF_OK : DCF_ECUDA;
}

int launch_hex_decode(const char* in, uint64_t nchars, void* out, dcf_status* status, cudaStream_t st) {
  if (nchars & 1) return DCF_EPARSE;
  const uint64_t nbytes = nchars / 2;
  const int vec = (((uintptr_t)in & 15) == 0 && ((uintptr_t)out & 7) == 0);
  const uint64_t need = (nbytes / 8 + 255) / 256 + 1;
  const int sms = sm_count();
  const unsigned g = (unsigned)(need < (uint64_t)sms * 8 ? need : (uint64_t)sms * 8);
  note_launch();
  hex_decode_kernel<<<g, 256, 0, st>>>(in, nbytes, (uint8_t*)out, status, vec);
  return cudaPeekAtLastError() == cudaSuccess ? DCF_OK : DCF_ECUDA;
}

int launch_hex_decode_pieces(const dcf_hex_piece* pieces, size_t n, uint64_t max_nchars, dcf_status* st,
                             cudaStream_t s) {
  if (n == 0) return DCF_OK;
  // Blocks per piece: enough for the longest, at most 64; pieces go along y
  // in launches of at most 65535.
  const uint64_t vecs = max_nchars / 16 + 1;
  const unsigned gx = (unsigned)std::max<uint64_t>(1, std::min<uint64_t>(4096, (vecs + 4 * 256 - 1) / (4 * 256)));
  for (size_t at = 0; at < n; at += 65535) {
    const unsigned gy = (unsigned)std::min<size_t>(65535, n - at);
    note_launch();
    hex_decode_pieces_kernel<<<dim3(gx, gy), 256, 0, s>>>(pieces + at, st);
    if (cudaPeekAtLastError() != cudaSuccess) return DCF_ECUDA;
  }
  return DCF_OK;
}

// ------------------------------------------------------------ byte hash

// A 64-bit hash of a byte range for constant deduplication: the sum over
// its 8-byte words (the last one zero-padded) of mix(word ^ index * phi),
// plus mix(length).  A sum of independent mixes reduces in any order, so
// every thread, warp and block adds its part with one atomicAdd.  mix is
// the SplitMix64 finaliser.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void __launch_bounds__(256) hash_pieces_kernel(const dcf_hash_piece* __restrict__ pieces,
                                                          unsigned long long* __restrict__ out) {
  const dcf_hash_piece pc = pieces[blockIdx.y];
  const uint64_t nw = pc.nbytes / 8, stride = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const uint8_t* b = (const uint8_t*)pc.data;
  const bool aligned = ((uintptr_t)b & 7) == 0;
  uint64_t h = 0;
  for (uint64_t i = tid; i < nw; i += stride) {
    uint64_t w;
    if (aligned) {
      w = __ldg((const unsigned long long*)b + i);
    } else {
      w = 0;
      for (int k = 0; k < 8; k++) w |= (uint64_t)b[8 * i + k] << (8 * k);
    }
    h += mix64(w ^ (i * 0x9E3779B97F4A7C15ull));
  }
  if (tid == 0) {
    uint64_t w = 0;
    for (uint64_t k = nw * 8; k < pc.nbytes; k++) w |= (uint64_t)b[k] << (8 * (k - nw * 8));
    if (pc.nbytes % 8) h += mix64(w ^ (nw * 0x9E3779B97F4A7C15ull));
    h += mix64(pc.nbytes);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) h += __shfl_xor_sync(0xFFFFFFFFu, h, o);
  if ((threadIdx.x & 31) == 0) atomicAdd(out + blockIdx.y, (unsigned long long)h);
}

int launch_hash_pieces(const dcf_hash_piece* pieces, size_t n, uint64_t max_bytes, uint64_t* out, cudaStream_t s) {
  if (n == 0) return DCF_OK;
  if (cudaMemsetAsync(out, 0, n * sizeof(uint64_t), s) != cudaSuccess) return DCF_ECUDA;
  // about 16 words per thread on the longest piece
  const uint64_t words = max_bytes / 8 + 1;
  const unsigned gx = (unsigned)std::max<uint64_t>(1, std::min<uint64_t>(4096, (words + 16 * 256 - 1) / (16 * 256)));
  for (size_t at = 0; at < n; at += 65535) {
    const unsigned gy = (unsigned)std::min<size_t>(65535, n - at);
    note_launch();
    hash_pieces_kernel<<<dim3(gx, gy), 256, 0, s>>>(pieces + at, (unsigned long long*)out + at);
    if (cudaPeekAtLastError() != cudaSuccess) return DCF_ECUDA;
  }
  return DCF_OK;
}

// --------------------------------------------------------------- select

// Folder::select on three dense constants (src/patterns/arith/canonicalize.rs:869-875):
// out[i] = cond[i] != 0 ? t[i] : f[i], a splat operand broadcast.  Chunks
// of 16 elements: one 16-byte load of conditions and 16-byte loads of each
// value operand, when every streamed pointer is 16-byte aligned (VEC).
template <typename T, bool VEC>
__global__ void __launch_bounds__(256) select_kernel(const uint8_t* __restrict__ c, int cs, const T* __restrict__ t,
                                                     int ts, const T* __restrict__ f, int fs, uint64_t n,
                                                     T* __restrict__ o, dcf_status* st) {
  constexpr int K = 16;
  constexpr int TV = K * (int)sizeof(T) / 16;  // 16-byte vectors per operand chunk
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const uint8_t c0 = c[0];
  const T t0 = t[0], f0 = f[0];
  const T o0 = c0 ? t0 : f0;
  bool nonsplat = false;
  const uint64_t chunks = VEC ? n / K : 0;
  for (uint64_t ch = tid; ch < chunks; ch += stride) {
    uint8_t cv[K];
    T tv[K], fv[K], ov[K];
    if (cs) {
#pragma unroll
      for (int k = 0; k < K; k++) cv[k] = c0;
    } else {
      *(uint4*)cv = __ldg((const uint4*)(c + ch * K));
    }
    if (ts) {
#pragma unroll
      for (int k = 0; k < K; k++) tv[k] = t0;
    } else {
#pragma unroll
      for (int j = 0; j < TV; j++) ((uint4*)tv)[j] = __ldg((const uint4*)(t + ch * K) + j);
    }
    if (fs) {
#pragma unroll
      for (int k = 0; k < K; k++) fv[k] = f0;
    } else {
#pragma unroll
      for (int j = 0; j < TV; j++) ((uint4*)fv)[j] = __ldg((const uint4*)(f + ch * K) + j);
    }
#pragma unroll
    for (int k = 0; k < K; k++) {
      ov[k] = cv[k] ? tv[k] : fv[k];
      nonsplat |= ov[k] != o0;
    }
#pragma unroll
    for (int j = 0; j < TV; j++) ((uint4*)(o + ch * K))[j] = ((const uint4*)ov)[j];
  }
  for (uint64_t i = chunks * K + tid; i < n; i += stride) {
    const T v = c[cs ? 0 : i] ? t[ts ? 0 : i] : f[fs ? 0 : i];
    o[i] = v;
    nonsplat |= v != o0;
  }
  report(st, ~0ull, nonsplat);
}

template <typename T>
static int select_t(const void* c, int cs, const void* t, int ts, const void* f, int fs, uint64_t n, void* o,
                    dcf_status* st, cudaStream_t s) {
  auto al = [](const void* p, int splat) { return splat || ((uintptr_t)p & 15) == 0; };
  const bool vec = al(c, cs) && al(t, ts) && al(f, fs) && al(o, 0);
  const uint64_t need = ((vec ? n / 16 : n) + 255) / 256 + 1;
  const int sms = sm_count();
  const unsigned g = (unsigned)(need < (uint64_t)sms * 8 ? need : (uint64_t)sms * 8);
  note_launch();
  if (vec)
    select_kernel<T, true><<<g, 256, 0, s>>>((const uint8_t*)c, cs, (const T*)t, ts, (const T*)f, fs, n, (T*)o, st);
  else
    select_kernel<T, false><<<g, 256, 0, s>>>((const uint8_t*)c, cs, (const T*)t, ts, (const T*)f, fs, n, (T*)o, st);
  return cudaPeekAtLastError() == cudaSuccess ? DCF_OK : DCF_ECUDA;
}

int launch_select(size_t es, const void* c, int cs, const void* t, int ts, const void* f, int fs, uint64_t n, void* o,
                  dcf_status* st, cudaStream_t s) {
  if (n == 0) return DCF_OK;
  switch (es) {
    case 1: return select_t<uint8_t>(c, cs, t, ts, f, fs, n, o, st, s);
    case 2: return select_t<uint16_t>(c, cs, t, ts, f, fs, n, o, st, s);
    case 4: return select_t<uint32_t>(c, cs, t, ts, f, fs, n, o, st, s);
    case 8: return select_t<uint64_t>(c, cs, t, ts, f, fs, n, o, st, s);
    default: return DCF_EINVAL;
  }
}

// ----------------------------------------------------------- splat test

template <typename T>
__global__ void __launch_bounds__(256) splat_kernel(const T* __restrict__ in, uint64_t n, dcf_status* st) {
  const T first = in[0];
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  bool differ = false;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) differ |= (in[i] != first);
  report(st, ~0ull, differ);
}

int launch_splat_check(const void* in, size_t es, uint64_t n, dcf_status* status, cudaStream_t st) {
  if (n == 0) return DCF_OK;
  const int sms = sm_count();
  const uint64_t need = (n + 255) / 256;
  const unsigned g = (unsigned)(need < (uint64_t)sms * 8 ? need : (uint64_t)sms * 8);
  note_launch();
  switch (es) {
    case 1: splat_kernel<uint8_t><<<g, 256, 0, st>>>((const uint8_t*)in, n, status); break;
    case 2: splat_kernel<uint16_t><<<g, 256, 0, st>>>((const uint16_t*)in, n, status); break;
    case 4: splat_kernel<uint32_t><<<g, 256, 0, st>>>((const uint32_t*)in, n, status); break;
    case 8: splat_kernel<uint64_t><<<g, 256, 0, st>>>((const uint64_t*)in, n, status); break;
    default: return DCF_EINVAL;
  }
  return cudaPeekAtLastError() == cudaSuccess ? DCF_OK : DCF_ECUDA;
}

}  // namespace dcf
