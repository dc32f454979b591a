// dcf_transpose_tma.cu — the layerwise transpose fold of 2-byte elements
// (bf16 / f16 / i16) as a bulk-tensor (TMA) pipeline.
//
// A rows x cols row-major matrix is cut into 64 x 64 tiles.  Persistent
// CTAs walk the tiles; each tile arrives in shared memory by one
// cp.async.bulk.tensor.2d load (a 64-element = 128-byte inner box with the
// 128-byte swizzle) on a four-stage mbarrier pipeline, so the next tiles
// are in flight while this one is written out.  Eight lanes read an 8 x 8 block
// as eight 16-byte rows (the swizzle puts the eight rows of a block in
// eight different bank groups, so the reads are conflict-free), transpose
// it in registers with three butterfly rounds of warp shuffles, and each
// lane stores one 16-byte output vector: a warp writes 64 contiguous bytes
// into each of eight output rows.  Waits are bounded; a CTA that gives up
// sets the status's error word, drains its copies and exits.
#include <cuda.h>

#include <mutex>

#include "dcf_kernels.cuh"

namespace dcf {

namespace {

constexpr int kT = 64;                        // tile side (elements)
constexpr int kTileBytes2 = kT * kT * 2;      // 8 KiB
constexpr int kStages2 = 4;

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_addr(dst)), "l"((uint64_t)map), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// 8 x 8 transpose of 16-bit elements over the 8 lanes of a group: lane i
// holds row i as four words (w[m] = e[i][2m] | e[i][2m+1] << 16) and ends
// holding column i the same way.
__device__ __forceinline__ void transpose8x8(uint32_t (&w)[4], int i) {
  const unsigned full = 0xFFFFFFFFu;
  {  // 4x4 blocks: the upper-right and lower-left blocks trade places
    const bool up = (i & 4) != 0;
    const uint32_t x = up ? w[0] : w[2], y = up ? w[1] : w[3];
    const uint32_t rx = __shfl_xor_sync(full, x, 4), ry = __shfl_xor_sync(full, y, 4);
    if (up) {
      w[0] = rx;
      w[1] = ry;
    } else {
      w[2] = rx;
      w[3] = ry;
    }
  }
#pragma unroll
  for (int h = 0; h < 2; h++) {  // 2x2 blocks inside each 4-wide half
    const bool up = (i & 2) != 0;
    const uint32_t x = up ? w[2 * h] : w[2 * h + 1];
    const uint32_t r = __shfl_xor_sync(full, x, 2);
    if (up) w[2 * h] = r;
    else w[2 * h + 1] = r;
  }
#pragma unroll
  for (int m = 0; m < 4; m++) {  // single elements inside each word
    const uint32_t r = __shfl_xor_sync(full, w[m], 1);
    w[m] = (i & 1) ? __byte_perm(r, w[m], 0x7632) : __byte_perm(w[m], r, 0x5410);
  }
}

__global__ void __launch_bounds__(256) transpose2_tma_kernel(const __grid_constant__ CUtensorMap map,
                                                             uint16_t* __restrict__ out, uint64_t rows,
                                                             uint64_t cols, dcf_status* st) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // The 128-byte swizzle repeats every 1024 bytes: stage buffers start on
  // a 1024-byte boundary.
  uint8_t* tiles = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(tiles + kStages2 * kTileBytes2);
  const uint64_t tr = (rows + kT - 1) / kT, tc = (cols + kT - 1) / kT, ntiles = tr * tc;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages2; s++) mbar_init(&full[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    for (int s = 0; s < kStages2; s++) {
      const uint64_t t = blockIdx.x + (uint64_t)s * gridDim.x;
      if (t < ntiles) {
        mbar_expect_tx(&full[s], kTileBytes2);
        tma_load_2d(tiles + s * kTileBytes2, &map, (int)((t % tc) * kT), (int)((t / tc) * kT), &full[s]);
      }
    }
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane >> 3, i = lane & 7;
  const int c = warp;  // the 16-byte column chunk (8 columns) this warp transposes
  uint64_t it = 0;
  bool dead = false;
  for (uint64_t t = blockIdx.x; t < ntiles; t += gridDim.x, it++) {
    const int s = (int)(it % kStages2);
    const bool ok = mbar_wait_bounded(&full[s], (unsigned)((it / kStages2) & 1));
    if (__syncthreads_or(!ok)) {
      dead = true;
      break;
    }
    const uint8_t* tile = tiles + s * kTileBytes2;
    const uint64_t r0 = (t / tc) * kT, c0 = (t % tc) * kT;
#pragma unroll
    for (int pass = 0; pass < 2; pass++) {
      const int rb = grp + 4 * pass;   // 8-row block
      const int row = rb * 8 + i;      // this lane's tile row
      const uint4 v = *(const uint4*)(tile + row * 128 + ((c ^ (row & 7)) << 4));
      uint32_t w[4] = {v.x, v.y, v.z, v.w};
      transpose8x8(w, i);
      // lane i now holds input column c*8+i, input rows rb*8 .. rb*8+7
      const uint64_t orow = c0 + (uint64_t)c * 8 + i, ocol = r0 + (uint64_t)rb * 8;
      if (orow < cols) {
        uint16_t* dst = out + orow * rows + ocol;
        if (ocol + 8 <= rows) {
          *(uint4*)dst = make_uint4(w[0], w[1], w[2], w[3]);
        } else {
          for (int k = 0; k < 8 && ocol + k < rows; k++) dst[k] = (uint16_t)(w[k >> 1] >> ((k & 1) * 16));
        }
      }
    }
    __syncthreads();  // every thread has read stage s
    if (threadIdx.x == 0) {
      const uint64_t tn = t + (uint64_t)kStages2 * gridDim.x;
      if (tn < ntiles) {
        mbar_expect_tx(&full[s], kTileBytes2);
        tma_load_2d(tiles + s * kTileBytes2, &map, (int)((tn % tc) * kT), (int)((tn / tc) * kT), &full[s]);
      }
    }
  }
  if (dead) {
    for (uint64_t j = it; j < it + kStages2; j++) {
      if (blockIdx.x + j * gridDim.x >= ntiles) break;
      mbar_wait_bounded(&full[j % kStages2], (unsigned)((j / kStages2) & 1));
    }
    if (threadIdx.x == 0 && st) atomicExch(&st->error, 1u);
  }
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiled)p;
    cudaGetLastError();
  });
  return fn;
}

}  // namespace

int launch_transpose2_tma(const void* in, void* out, uint64_t rows, uint64_t cols, dcf_status* st,
                          cudaStream_t s) {
  // The tensor map needs a 16-byte aligned base and a row pitch that is a
  // multiple of 16 bytes; the 16-byte output stores need the same of the
  // output.  Coordinates are 32-bit.
  if (((uintptr_t)in & 15) || ((uintptr_t)out & 15) || cols % 8 || rows % 8 || rows == 0 || cols == 0 ||
      rows >= (1ull << 31) || cols >= (1ull << 31))
    return DCF_EUNSUPPORTED;
  EncodeTiled enc = encoder();
  if (!enc) return DCF_EUNSUPPORTED;
  CUtensorMap map;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {kT, kT};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(in), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return DCF_EUNSUPPORTED;
  const int smem = kStages2 * kTileBytes2 + 1024 + kStages2 * 8;
  if (!prepare_smem((const void*)transpose2_tma_kernel, smem)) return DCF_ECUDA;
  const uint64_t ntiles = ((rows + kT - 1) / kT) * ((cols + kT - 1) / kT);
  const int sms = sm_count_current();
  const uint64_t g = ntiles < (uint64_t)sms * 6 ? ntiles : (uint64_t)sms * 6;
  note_launch();
  transpose2_tma_kernel<<<(unsigned)g, 256, smem, s>>>(map, (uint16_t*)out, rows, cols, st);
  return cudaPeekAtLastError() == cudaSuccess ? DCF_OK : DCF_ECUDA;
}

}  // namespace dcf
