// st_umma.cuh -- fifth-generation tensor-core (tcgen05) building blocks for
// sm_100a: tensor-memory allocation, the kind::f16 MMA with both operands in
// shared memory and the accumulator in tensor memory, completion through
// mbarriers, and the tensor-memory loads of the epilogue. Hand-written PTX.
//
// Operand layout: "no swizzle, K-major" core matrices. A core matrix is 8 rows
// x 16 bytes (8 bf16/fp16 elements of K, or 4 tf32), stored as 128 contiguous
// bytes. A tile of R rows x 128 bytes of K (64 16-bit or 32 tf32 elements) is
// stored as [R/8 row groups][8 K groups][8 rows][16 bytes] so that, in the
// shared-memory descriptor, the K-adjacent core matrices are 128 bytes apart
// (leading-dimension byte offset) and the row-group-adjacent ones 1024 bytes
// apart (stride-dimension byte offset). One MMA consumes 32 bytes of K (two
// core matrices: K = 16 of kind::f16, K = 8 of kind::tf32); the next starts
// 256 bytes further.
//
// fp32 GEMMs run as three TF32 products ("3xTF32"): each operand x is split
// into hi = tf32(x) and lo = tf32(x - hi), and A B = Ahi Bhi + Ahi Blo +
// Alo Bhi accumulates in fp32; the dropped Alo Blo and the rounding of lo are
// about 2^-22 of each product, below fp32's own accumulation error at these
// lengths.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "st_ring.cuh"

namespace st {

constexpr int kUmmaM = 128;          // rows of A (weight rows) per MMA tile
constexpr int kUmmaK = 16;           // K per MMA instruction (16-bit operands)
constexpr int kTileK = 64;           // K per staged chunk (four MMAs), 16-bit operands
constexpr int kTileK32 = 32;         // K per staged chunk, tf32 operands
constexpr unsigned kCoreBytes = 128; // one 8 x 16-byte core matrix
constexpr unsigned kLbo = 128;       // K-adjacent core matrices
constexpr unsigned kSbo = 1024;      // row-group-adjacent core matrices (8 K groups of 128 bytes)

// Element offset of (row r, column k) in the tiled layout of a matrix whose
// tiles hold `tile_rows` rows (a multiple of 8) and 64 columns, tiles ordered
// [row tile][K chunk] with `kchunks` chunks per row tile.
__host__ __device__ inline size_t umma_tile_offset(size_t r, size_t k, size_t tile_rows, size_t kchunks) {
  const size_t tile = (r / tile_rows) * kchunks + k / kTileK;
  const size_t rr = r % tile_rows;
  return tile * tile_rows * kTileK + (((rr >> 3) * 8 + ((k >> 3) & 7)) * 64) + (rr & 7) * 8 + (k & 7);
}

// Offset of (stream s, column k) in the tiled B operand (one tile of all
// `spad` rows per 64-column chunk; s < spad): 32-bit arithmetic, no division.
__host__ __device__ __forceinline__ unsigned z_tile_offset(unsigned s, unsigned k, unsigned spad) {
  return (k >> 6) * (spad << 6) + ((((s >> 3) << 3) + ((k >> 3) & 7u)) << 6) + ((s & 7u) << 3) + (k & 7u);
}
// The same for 32-bit elements (32 columns per chunk).
__host__ __device__ __forceinline__ unsigned z_tile_offset32(unsigned s, unsigned k, unsigned spad) {
  return (k >> 5) * (spad << 5) + ((((s >> 3) << 3) + ((k >> 2) & 7u)) << 5) + ((s & 7u) << 2) + (k & 3u);
}

// The same layout for 32-bit elements (tf32 operands, 32 columns per tile).
__host__ __device__ inline size_t umma_tile_offset32(size_t r, size_t k, size_t tile_rows, size_t kchunks) {
  const size_t tile = (r / tile_rows) * kchunks + k / kTileK32;
  const size_t rr = r % tile_rows;
  return tile * tile_rows * kTileK32 + (((rr >> 3) * 8 + ((k >> 2) & 7)) * 32) + (rr & 7) * 4 + (k & 3);
}

// x rounded to tf32 (10 explicit mantissa bits, nearest, ties away from zero),
// as an fp32 bit pattern whose low 13 bits are zero.
__device__ __forceinline__ float to_tf32(float x) {
  unsigned r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Shared-memory matrix descriptor (tcgen05 format): start address >> 4 in
// bits 0-13, leading-dimension byte offset >> 4 in 16-29, stride-dimension
// byte offset >> 4 in 32-45, descriptor version 1 in bits 46-47, base offset
// 0, no swizzle (bits 61-63 = 0).
__device__ __forceinline__ unsigned long long umma_desc(const void* smem) {
  const unsigned addr = smem_addr(smem);
  return (unsigned long long)((addr & 0x3FFFFu) >> 4) | ((unsigned long long)(kLbo >> 4) << 16) |
         ((unsigned long long)(kSbo >> 4) << 32) | (1ull << 46);
}

// Instruction descriptor of kind::f16 / kind::tf32: fp32 accumulator (bits
// 4-5 = 1), A and B both bf16 (bits 7-9 and 10-12 = 1), both fp16 (0) or both
// tf32 (2, for fp32 storage), both K-major (bits 15, 16 = 0), N >> 3 in bits
// 17-22, M >> 4 in bits 24-28.
template <typename T>
__device__ __forceinline__ unsigned umma_idesc(int m, int n) {
  const unsigned ab = std::is_same<T, __nv_bfloat16>::value ? 1u : std::is_same<T, float>::value ? 2u : 0u;
  return (1u << 4) | (ab << 7) | (ab << 10) | ((unsigned)(n >> 3) << 17) | ((unsigned)(m >> 4) << 24);
}

// Tensor memory: allocated by one whole warp; the base address lands in *dst.
__device__ __forceinline__ void tmem_alloc(unsigned* dst, unsigned ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(unsigned taddr, unsigned ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D (tensor memory) = A B^T (+ D when `accumulate`), issued by one thread.
__device__ __forceinline__ void umma_f16(unsigned d_tmem, unsigned long long adesc, unsigned long long bdesc,
                                         unsigned idesc, unsigned accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The same with tf32 operands (kind::tf32, K = 8 per instruction).
__device__ __forceinline__ void umma_tf32(unsigned d_tmem, unsigned long long adesc, unsigned long long bdesc,
                                          unsigned idesc, unsigned accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// One arrival on `bar` once every MMA this thread issued so far has completed
// (its shared-memory operands may then be overwritten, its accumulator read).
__device__ __forceinline__ void umma_commit(unsigned long long* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

// 32 lanes x 16 columns of 32-bit accumulator: thread i of the warp receives
// lane (taddr's lane + i), columns [col, col + 16). Waits for the load.
__device__ __forceinline__ void tmem_ld16(unsigned taddr, float (&v)[16]) {
  unsigned r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Bounded wait on an mbarrier phase; false when `timeout_ns` ran out.
__device__ __forceinline__ bool mbar_wait_bounded(unsigned long long* bar, unsigned parity,
                                                  unsigned long long timeout_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long start = globaltimer();
  while (!mbar_try_wait_for(bar, parity, 1000u))
    if (globaltimer() - start > timeout_ns) return false;
  return true;
}

}  // namespace st
