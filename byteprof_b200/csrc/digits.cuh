// Activations as exact signed base-256 digit planes, the A or B operand of the integer MMA (kind::i8)
// used by the int8 and int4 skinny kernels.
//
// Per activation row m, e_m = exponent of max_k |x[m, k]| and x = X 2^(e_m - 29) with |X| < 2^30: bf16
// values down to 2^-22 of the row maximum are exact, smaller ones are rounded to the nearest multiple of
// 2^(e_m - 29) (an error below 2^-29 of the row maximum). X = d0 + 2^8 d1 + 2^16 d2 + 2^24 d3 with every
// d_p in [-128, 127]; plane p of row m is row 4 m + p of the [4 M, K] digit matrix.
#pragma once

#include <stdint.h>

namespace bp {

constexpr int kDigitPlanes = 4;
constexpr int kFracBits = 29;
constexpr int kNonFinite = 0x7fffffff;  // row exponent marker: the row holds an Inf or a NaN

// Exponent e with 2^e <= max|x| < 2^(e+1) from the largest |x| bit pattern of a bf16 row.
__device__ __forceinline__ int row_exponent(uint32_t amax_bits) {
  if (amax_bits >= 0x7f80u) return kNonFinite;
  if (amax_bits == 0) return 0;
  const int ef = static_cast<int>(amax_bits >> 7);
  return ef == 0 ? -127 : ef - 127;  // subnormal maximum: 2^-127 bounds it from above by 2^-126
}

// X = x / 2^(e - 29) rounded to nearest (ties to even) for one bf16 bit pattern; |X| < 2^30.
__device__ __forceinline__ int fixed_point(uint32_t b, int e) {
  const int ef = static_cast<int>((b >> 7) & 0xffu);
  int mant = static_cast<int>(b & 0x7fu);
  int f = -126;
  if (ef != 0) {
    mant |= 0x80;
    f = ef - 127;
  }
  const int sh = f - e + (kFracBits - 7);  // x = mant * 2^(f - 7) = mant * 2^sh * 2^(e - 29); sh <= 23
  int X;
  if (sh >= 0) {
    X = mant << sh;
  } else {
    const int r = -sh;
    X = r >= 9 ? 0 : (mant + (1 << (r - 1)) - 1 + ((mant >> r) & 1)) >> r;  // mant < 2^8: r >= 9 rounds to 0
  }
  return (b & 0x8000u) ? -X : X;
}

// 8 bf16 activations (one 16-byte chunk) -> 8 bytes of each of the 4 digit planes (|X| < 2^30 keeps d3
// within [-64, 64]); returns the exact sum of the 8 fixed-point values X.
__device__ __forceinline__ long long digitise8(const uint4& v, int e, uint32_t (&pl)[kDigitPlanes][2]) {
  const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
  long long sum = 0;
#pragma unroll
  for (int p = 0; p < kDigitPlanes; ++p) pl[p][0] = pl[p][1] = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int X = fixed_point((wv[j >> 1] >> (16 * (j & 1))) & 0xffffu, e);
    sum += X;
    const int d0 = static_cast<int>(static_cast<int8_t>(X & 0xff));
    const int r1 = (X - d0) >> 8;
    const int d1 = static_cast<int>(static_cast<int8_t>(r1 & 0xff));
    const int r2 = (r1 - d1) >> 8;
    const int d2 = static_cast<int>(static_cast<int8_t>(r2 & 0xff));
    const int d3 = (r2 - d2) >> 8;
    const int sh = 8 * (j & 3);
    pl[0][j >> 2] |= (static_cast<uint32_t>(d0) & 0xffu) << sh;
    pl[1][j >> 2] |= (static_cast<uint32_t>(d1) & 0xffu) << sh;
    pl[2][j >> 2] |= (static_cast<uint32_t>(d2) & 0xffu) << sh;
    pl[3][j >> 2] |= (static_cast<uint32_t>(d3) & 0xffu) << sh;
  }
  return sum;
}

}  // namespace bp
