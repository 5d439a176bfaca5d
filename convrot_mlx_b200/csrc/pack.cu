// Signed int4 packing kernels: unpack (core.py:108-120, Metal core.py:915-922),
// pack (core.py:97-105) and the lossless NK <-> KN repack (core.py:123-146).
#include "common.cuh"

namespace convrot {

// 8 packed bytes -> 16 int8 values per thread.
__global__ void unpack_int4_kernel(const uint8_t* __restrict__ in, int64_t n_bytes, int8_t* __restrict__ out) {
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (i + 8 <= n_bytes) {
    const uint2 w = *reinterpret_cast<const uint2*>(in + i);
    uint32_t src[2] = {w.x, w.y};
    uint32_t dst[4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      // nibbles -> sign-extended bytes: low nibbles at even, high at odd positions
      const uint32_t lo = src[j] & 0x0F0F0F0Fu;
      const uint32_t hi = (src[j] >> 4) & 0x0F0F0F0Fu;
      const uint32_t los = lo | ((lo & 0x08080808u) * 0x1Eu);  // 0x08 * 0x1E = 0xF0: fill the sign
      const uint32_t his = hi | ((hi & 0x08080808u) * 0x1Eu);
      dst[2 * j] = __byte_perm(los, his, 0x5140);
      dst[2 * j + 1] = __byte_perm(los, his, 0x7362);
    }
    *reinterpret_cast<uint4*>(out + 2 * i) = make_uint4(dst[0], dst[1], dst[2], dst[3]);
  } else {
    for (int64_t b = i; b < n_bytes; ++b) {
      const int lo = in[b] & 0xF, hi = (in[b] >> 4) & 0xF;
      out[2 * b] = static_cast<int8_t>(lo >= 8 ? lo - 16 : lo);
      out[2 * b + 1] = static_cast<int8_t>(hi >= 8 ? hi - 16 : hi);
    }
  }
}

// 16 int8 values -> 8 packed bytes per thread.
__global__ void pack_int4_kernel(const int8_t* __restrict__ in, int64_t n_values, uint8_t* __restrict__ out) {
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 16;
  if (i + 16 <= n_values) {
    const uint4 w = *reinterpret_cast<const uint4*>(in + i);
    const uint32_t src[4] = {w.x, w.y, w.z, w.w};
    uint32_t dst[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint32_t a = src[2 * j] & 0x0F0F0F0Fu, b = src[2 * j + 1] & 0x0F0F0F0Fu;
      // bytes (e0,e1,e2,e3) -> (e0 | e1<<4, e2 | e3<<4)
      const uint32_t a2 = (a | (a >> 4)) & 0x00FF00FFu;  // byte0 = e0|e1<<4, byte2 = e2|e3<<4
      const uint32_t b2 = (b | (b >> 4)) & 0x00FF00FFu;
      dst[j] = __byte_perm(a2, b2, 0x6420);
    }
    *reinterpret_cast<uint2*>(out + i / 2) = make_uint2(dst[0], dst[1]);
  } else {
    for (int64_t v = i; v + 1 < n_values; v += 2) {
      out[v / 2] = static_cast<uint8_t>((in[v] & 0xF) | ((in[v + 1] & 0xF) << 4));
    }
  }
}

// out (C2 = 2*packed_cols rows, R/2 bytes) from in (R rows, packed_cols bytes):
// out element (j, i) = in element (i, j).  A 64 (i) x 64 (j) tile per block.
__global__ void repack_transpose_kernel(const uint8_t* __restrict__ in, int64_t R, int64_t packed_cols,
                                        uint8_t* __restrict__ out) {
  __shared__ uint8_t tile[64][65];  // [j][i] nibbles
  const int64_t i0 = static_cast<int64_t>(blockIdx.y) * 64;
  const int64_t j0 = static_cast<int64_t>(blockIdx.x) * 64;
  const int64_t C2 = packed_cols * 2;
  const int tx = threadIdx.x;  // 0..31 -> packed byte column within the tile
  for (int r = threadIdx.y; r < 64; r += blockDim.y) {
    const int64_t i = i0 + r;
    const int64_t jb = j0 / 2 + tx;
    uint8_t v = 0;
    if (i < R && jb < packed_cols) v = in[i * packed_cols + jb];
    tile[2 * tx][r] = v & 0xF;
    tile[2 * tx + 1][r] = (v >> 4) & 0xF;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 64; r += blockDim.y) {
    const int64_t j = j0 + r;
    const int64_t ob = i0 / 2 + tx;
    if (j < C2 && 2 * ob < R) out[j * (R / 2) + ob] = static_cast<uint8_t>(tile[r][2 * tx] | (tile[r][2 * tx + 1] << 4));
  }
}

}  // namespace convrot

extern "C" {

int convrot_unpack_int4(const uint8_t* packed, int64_t n_bytes, int8_t* out, void* stream) {
  CONVROT_REQUIRE(n_bytes >= 0, CONVROT_ERR_INVALID, "negative size");
  if (n_bytes == 0) return CONVROT_OK;
  CONVROT_REQUIRE(packed && out, CONVROT_ERR_INVALID, "null pointer");
  CONVROT_REQUIRE(convrot::aligned_to(packed, 8) && convrot::aligned_to(out, 16), CONVROT_ERR_INVALID,
                  "unpack needs 8-byte aligned input and 16-byte aligned output");
  const int64_t threads = (n_bytes + 7) / 8;
  const int block = 256;
  const int64_t grid = (threads + block - 1) / block;
  CONVROT_REQUIRE(grid < 2147483647LL, CONVROT_ERR_UNSUPPORTED, "tensor too large");
  convrot::unpack_int4_kernel<<<static_cast<unsigned>(grid), block, 0, static_cast<cudaStream_t>(stream)>>>(packed, n_bytes, out);
  return convrot::check_launch("unpack_int4");
}

int convrot_pack_int4(const int8_t* values, int64_t n_values, uint8_t* out, void* stream) {
  CONVROT_REQUIRE(n_values >= 0 && n_values % 2 == 0, CONVROT_ERR_INVALID, "last dimension must be even, got %lld",
                  static_cast<long long>(n_values));
  if (n_values == 0) return CONVROT_OK;
  CONVROT_REQUIRE(values && out, CONVROT_ERR_INVALID, "null pointer");
  CONVROT_REQUIRE(convrot::aligned_to(values, 16) && convrot::aligned_to(out, 8), CONVROT_ERR_INVALID,
                  "pack needs 16-byte aligned input and 8-byte aligned output");
  const int64_t threads = (n_values + 15) / 16;
  const int block = 256;
  const int64_t grid = (threads + block - 1) / block;
  CONVROT_REQUIRE(grid < 2147483647LL, CONVROT_ERR_UNSUPPORTED, "tensor too large");
  convrot::pack_int4_kernel<<<static_cast<unsigned>(grid), block, 0, static_cast<cudaStream_t>(stream)>>>(values, n_values, out);
  return convrot::check_launch("pack_int4");
}

int convrot_repack_int4_transpose(const uint8_t* in, int64_t rows, int64_t packed_cols, uint8_t* out, void* stream) {
  CONVROT_REQUIRE(rows >= 0 && packed_cols >= 0, CONVROT_ERR_INVALID, "invalid shape");
  CONVROT_REQUIRE(rows % 2 == 0, CONVROT_ERR_INVALID, "int4 repacking requires an even row count, got %lld",
                  static_cast<long long>(rows));
  if (rows == 0 || packed_cols == 0) return CONVROT_OK;
  CONVROT_REQUIRE(in && out, CONVROT_ERR_INVALID, "null pointer");
  const int64_t gx = (2 * packed_cols + 63) / 64, gy = (rows + 63) / 64;
  CONVROT_REQUIRE(gx < 2147483647LL && gy < 65535, CONVROT_ERR_UNSUPPORTED, "tensor too large");
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy));
  convrot::repack_transpose_kernel<<<grid, dim3(32, 8), 0, static_cast<cudaStream_t>(stream)>>>(in, rows, packed_cols, out);
  return convrot::check_launch("repack_int4_transpose");
}

}  // extern "C"
