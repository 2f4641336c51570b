// gemv_core.cuh — the CUDA-core dequantising MAC shared by the streaming GEMV
// (gemv_q.cu) and the persistent decode chain (chain.cu).
//
// Dequantization costs one LOP3 + one FFMA per code. A code field masked in
// place, (word & (mask << pos)), read as an f32 bit pattern is the subnormal
// raw * 2^(pos-149); FFMA handles subnormal inputs at full rate and exactly.
// x is pre-scaled in shared memory by 2^(S - pos) (a power of two, exact) so
// every product equals x * raw * 2^(S-149) with a normal result. S is chosen
// per activation row from max|x| so nothing overflows. Offset-binary codes are
// accumulated as raw = q + zp; the caller subtracts the row mean of x first and
// corrects with mu * sum_k q and zp * sum_k (x - mu) in its epilogue.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace gqcore {

template <int BITS>
struct Fmt {
  static constexpr int kPerWord = 32 / BITS;      // codes per 32-bit word
  static constexpr int kPerChunk = 4 * kPerWord;  // codes per 16-byte chunk
  static constexpr int kPad = kPerChunk + 4;      // padded x floats per chunk
  static constexpr int kZp = 1 << (BITS - 1);     // offset-binary zero point
  // Codes [0, kSplit) are masked straight out of the word; the rest out of the
  // word shifted right by kShift, so every field stays inside f32 bits 0..22.
  static constexpr int kSplit = BITS == 4 ? 5 : (BITS == 2 ? 11 : 2);
  static constexpr int kShift = BITS == 4 ? 12 : 16;
};

// Bit position of code j of a word inside the 32-bit register it is masked from.
template <int BITS>
__host__ __device__ constexpr int code_pos(int j) {
  return j < Fmt<BITS>::kSplit ? j * BITS : j * BITS - Fmt<BITS>::kShift;
}

__device__ __forceinline__ float pow2f(int e) {  // exact 2^e for e in [-126, 127]
  return __int_as_float((e + 127) << 23);
}

// MAC of one 16-byte chunk (4 words) of NW weights against MT activation rows.
// acc[h][m][q]: ACC independent accumulators per (weight, row). Per word: one
// XOR (I8 sign flip to offset binary) and one shift; per code: one AND with an
// immediate mask and one FFMA per activation row.
template <int BITS, bool SIGNED, int MT, int NW, int ACC>
__device__ __forceinline__ void mac_chunk(const uint4 (&wv)[NW], const float *xc, int xs_mstride,
                                          float (&acc)[NW][MT][ACC]) {
  using F = Fmt<BITS>;
  constexpr uint32_t kMask = (1u << BITS) - 1u;
  constexpr uint32_t kXor = (BITS == 8 && SIGNED) ? 0x80808080u : 0u;
#pragma unroll
  for (int wi = 0; wi < 4; ++wi) {
    uint32_t lo[NW], hi[NW];
#pragma unroll
    for (int h = 0; h < NW; ++h) {
      lo[h] = (wi == 0 ? wv[h].x : wi == 1 ? wv[h].y : wi == 2 ? wv[h].z : wv[h].w) ^ kXor;
      hi[h] = lo[h] >> F::kShift;
    }
#pragma unroll
    for (int j4 = 0; j4 < F::kPerWord; j4 += 4) {
      float4 xv[MT];
#pragma unroll
      for (int m = 0; m < MT; ++m)
        xv[m] = *reinterpret_cast<const float4 *>(xc + m * xs_mstride + wi * F::kPerWord + j4);
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int j = j4 + jj;
#pragma unroll
        for (int h = 0; h < NW; ++h) {
          const float fld = __uint_as_float(((j < F::kSplit) ? lo[h] : hi[h]) & (kMask << code_pos<BITS>(j)));
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            const float xvj = jj == 0 ? xv[m].x : jj == 1 ? xv[m].y : jj == 2 ? xv[m].z : xv[m].w;
            acc[h][m][j % ACC] = __fmaf_rn(xvj, fld, acc[h][m][j % ACC]);
          }
        }
      }
    }
  }
}

}  // namespace gqcore
