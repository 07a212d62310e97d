// The repacked ("blob") weight layout and the int4 -> fp16/bf16 dequantisation
// shared by the repack, dequant and GEMM kernels.
//
// AWQ checkpoint layout (reference: layers/quantization/awq.py:87-124):
//   qweight int32 [K, N/8]   logical column 8j+i of packed word j sits at bits
//                            4*r(i) with r = [0,4,1,5,2,6,3,7]  (awq_triton.py:53-62)
//   qzeros  int32 [K/G, N/8] same packing
//   scales  fp16/bf16 [K/G, N]
//   W[k, n] = (q[k, n] - z[k/G, n]) * s[k/G, n], one rounding to the activation
//   dtype (awq_triton.py:119-122).
//
// Blob layout (this library's own):
//   The [K, N] weight is padded to Kp = roundup(K,128), Np = roundup(N,128) and
//   cut into blocks of 128 output features x 128 input features. Block (nt, kb)
//   starts at byte ((nt * KB) + kb) * block_bytes, so the blocks one output tile
//   needs along K are contiguous and stream with one bulk copy each.
//   Inside a block:
//     [0, 8192)            2048 words. Word (row r, j) holds k = 128kb + 8j + i,
//                          i = 0..7, of feature n = 128nt + r; it is stored at
//                          word index ((j/4)*128 + r)*4 + (j%4), so that 128
//                          threads reading row r with 16-byte loads hit distinct
//                          banks. Nibble for i = 2p is at bits [4p, 4p+4), for
//                          i = 2p+1 at bits [16+4p, 16+4p+4): a mask 0x000F000F
//                          yields the pair (i=2p, i=2p+1) as two 16-bit lanes.
//     [8192, +256*gpb)     scales, u16 index g*128 + r (g = group within block)
//     [.., +64*gpb)        zeros, u32 index g*16 + r/8, nibble 4*(r%8)
//   gpb = groups per block = 128/G for G in {32, 64}, else 1 (G a multiple of
//   128: the block holds the single group it lies in).
//   The number of k-blocks per feature tile is padded to an even count,
//   KB = 2 * ceil(K / 256), so that the GEMM can stream two blocks (256 k) per
//   pipeline stage with one bulk copy.
//   Padding features and padding K carry q = z = 0 and s = 0, i.e. weight 0.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace awqb {

constexpr int kBlockN = 128;        // output features per block / per MMA tile
constexpr int kBlockK = 128;        // input features per block / per pipeline stage
constexpr int kWordBytes = 8192;    // packed nibbles of one block

__host__ __device__ constexpr int64_t blob_kblocks(int64_t K) { return 2 * ((K + 2 * kBlockK - 1) / (2 * kBlockK)); }
__host__ __device__ constexpr int groups_per_block(int G) { return G < kBlockK ? kBlockK / G : 1; }
__host__ __device__ constexpr int block_bytes_for_gpb(int gpb) { return kWordBytes + 320 * gpb; }
__host__ __device__ constexpr int scale_off() { return kWordBytes; }
__host__ __device__ constexpr int zero_off(int gpb) { return kWordBytes + 256 * gpb; }
__host__ __device__ constexpr int word_index(int r, int j) { return (((j >> 2) * 128 + r) << 2) + (j & 3); }

template <typename T> struct DqTraits;

// fp16: lane values 1024 + q come from OR-ing the nibble into 0x6400; the
// second pair of a byte gives 1024 + 16q and is brought back with an exact FMA
// by 1/16. (q - z) is an exact small integer; the final multiply by the scale
// is the only rounding, as in the reference dequantisation.
template <> struct DqTraits<__half> {
  struct Terms { uint32_t zlo, zhi, s2; };
  __device__ __forceinline__ static Terms make(uint16_t scale_bits, uint32_t z) {
    Terms t;
    t.zlo = (0x6400u | z) * 0x00010001u;                 // (1024 + z) in both lanes
    __half zh = __float2half_rn(-(64.0f + (float)z));    // exact: integer <= 79
    uint16_t zb = __half_as_ushort(zh);
    t.zhi = (uint32_t)zb * 0x00010001u;
    t.s2 = (uint32_t)scale_bits * 0x00010001u;
    return t;
  }
  __device__ __forceinline__ static uint4 dq8(uint32_t w, const Terms& t) {
    uint32_t a0, a1, a2, a3;
    const uint32_t w8 = w >> 8;
    asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(a0) : "r"(w), "r"(0x000F000Fu), "r"(0x64006400u));
    asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(a1) : "r"(w), "r"(0x00F000F0u), "r"(0x64006400u));
    asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(a2) : "r"(w8), "r"(0x000F000Fu), "r"(0x64006400u));
    asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(a3) : "r"(w8), "r"(0x00F000F0u), "r"(0x64006400u));
    const __half2 zlo = *reinterpret_cast<const __half2*>(&t.zlo);
    const __half2 zhi = *reinterpret_cast<const __half2*>(&t.zhi);
    const __half2 s2 = *reinterpret_cast<const __half2*>(&t.s2);
    const __half2 sixteenth = __halves2half2(__ushort_as_half(0x2C00), __ushort_as_half(0x2C00));
    __half2 p0 = __hsub2(*reinterpret_cast<__half2*>(&a0), zlo);
    __half2 p1 = __hfma2(*reinterpret_cast<__half2*>(&a1), sixteenth, zhi);
    __half2 p2 = __hsub2(*reinterpret_cast<__half2*>(&a2), zlo);
    __half2 p3 = __hfma2(*reinterpret_cast<__half2*>(&a3), sixteenth, zhi);
    p0 = __hmul2(p0, s2);
    p1 = __hmul2(p1, s2);
    p2 = __hmul2(p2, s2);
    p3 = __hmul2(p3, s2);
    uint4 o;
    o.x = *reinterpret_cast<uint32_t*>(&p0);
    o.y = *reinterpret_cast<uint32_t*>(&p1);
    o.z = *reinterpret_cast<uint32_t*>(&p2);
    o.w = *reinterpret_cast<uint32_t*>(&p3);
    return o;
  }
};

// bf16: 0x4300 is 128.0 with a unit last place, so OR-ing a nibble into the
// mantissa gives 128 + q exactly. Subtracting (128 + z) is exact; the multiply
// by the scale is the only rounding.
template <> struct DqTraits<__nv_bfloat16> {
  struct Terms { uint32_t zb, s2; };
  __device__ __forceinline__ static Terms make(uint16_t scale_bits, uint32_t z) {
    Terms t;
    t.zb = (0x4300u | z) * 0x00010001u;
    t.s2 = (uint32_t)scale_bits * 0x00010001u;
    return t;
  }
  __device__ __forceinline__ static uint4 dq8(uint32_t w, const Terms& t) {
    uint32_t a0, a1, a2, a3;
    asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(a0) : "r"(w), "r"(0x000F000Fu), "r"(0x43004300u));
    asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(a1) : "r"(w >> 4), "r"(0x000F000Fu), "r"(0x43004300u));
    asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(a2) : "r"(w >> 8), "r"(0x000F000Fu), "r"(0x43004300u));
    asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(a3) : "r"(w >> 12), "r"(0x000F000Fu), "r"(0x43004300u));
    const __nv_bfloat162 zb = *reinterpret_cast<const __nv_bfloat162*>(&t.zb);
    const __nv_bfloat162 s2 = *reinterpret_cast<const __nv_bfloat162*>(&t.s2);
    __nv_bfloat162 p0 = __hmul2(__hsub2(*reinterpret_cast<__nv_bfloat162*>(&a0), zb), s2);
    __nv_bfloat162 p1 = __hmul2(__hsub2(*reinterpret_cast<__nv_bfloat162*>(&a1), zb), s2);
    __nv_bfloat162 p2 = __hmul2(__hsub2(*reinterpret_cast<__nv_bfloat162*>(&a2), zb), s2);
    __nv_bfloat162 p3 = __hmul2(__hsub2(*reinterpret_cast<__nv_bfloat162*>(&a3), zb), s2);
    uint4 o;
    o.x = *reinterpret_cast<uint32_t*>(&p0);
    o.y = *reinterpret_cast<uint32_t*>(&p1);
    o.z = *reinterpret_cast<uint32_t*>(&p2);
    o.w = *reinterpret_cast<uint32_t*>(&p3);
    return o;
  }
};

// Reads the scale bits and zero point of (group g, row r) from a block in
// shared or global memory.
__device__ __forceinline__ void block_scale_zero(const uint8_t* blk, int gpb, int g, int r,
                                                 uint16_t& s_bits, uint32_t& z) {
  s_bits = reinterpret_cast<const uint16_t*>(blk + scale_off())[g * 128 + r];
  const uint32_t zw = reinterpret_cast<const uint32_t*>(blk + zero_off(gpb))[g * 16 + (r >> 3)];
  z = (zw >> (4 * (r & 7))) & 0xFu;
}

}  // namespace awqb
