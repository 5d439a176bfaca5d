// Fused ConvRot activation preparation for sm_100a.
//
// One CTA owns one row.  The row is read from HBM exactly once (the reference
// Metal kernel, core.py:205-304, reads it twice: once for the absmax pass and
// once to re-rotate and quantize).  The rotated row waits in shared memory
// for the row absmax, then is quantized and written with 16-byte stores.
//
// Pair-words.  Element e of the first half of the row is paired with element
// e + half (half = ceil(groups / 2) * G), which sits at the same position of
// another Hadamard group.  No butterfly stage ever mixes the two, so every
// stage runs on packed bf16x2 / half2 words (two rows of the butterfly per
// instruction).  A thread works on "units" of 16 consecutive pair-words:
//   phase 1  global -> registers, butterfly strides 1 and 4 in registers
//   phase 2  (G >= 64) strides 16 and 64 over columns of shared memory
//   phase 3  (G == 1024) stride 256
//   quantize rotated pair-words -> codes, one 16-byte store per half-unit.
// Every add/sub is rounded to the input dtype in the reference's order
// (core.py:180-201: ((a+b)+c)-d, ((a+b)-c)+d, ((a-b)+c)+d, ((-a+b)+c)+d),
// then x / sqrt(G) (exact), scale = T(T(max(absmax, T(1e-10))) / 7) and
// code = clamp(rint(T(x / scale)), -7, 7) (core.py:149-158, :258-298).
#pragma once
#include <type_traits>

#include "common.cuh"

namespace convrot {

enum PrepMode : int { kModeI8 = 0, kModePacked = 1, kModeRotate = 2 };

// Word index of pair-element p in shared memory: rows of 32 words, 16-byte
// chunks XOR-swizzled so that the row-wise (phase 1 / quantize) and the
// column-wise (phases 2 and 3) accesses are all free of bank conflicts.
// swz(p) = p ^ (h(p) << 2) with h made of bit selections and XORs, so swz is
// linear over XOR: swz(a ^ b) == swz(a) ^ swz(b).  Every access below is a
// per-thread base plus a loop offset on disjoint bits (so + is ^), and its
// index is the thread's swizzled base XOR a compile-time constant.
__host__ __device__ constexpr int swz(int p) {
  const int r = p >> 5;
  const int h = (r & 3) | ((((r >> 1) ^ (r >> 3)) & 1) << 2);
  return (r << 5) | ((((p >> 2) & 7) ^ h) << 2) | (p & 3);
}

// One radix-4 butterfly on pair-words.  kExact keeps even the sign of a zero
// result identical to the reference ((-a) + b is computed as b - a); the
// quantizing modes use (c - (a - b)) + d instead, one op fewer, which can
// differ from it only in the sign of an exact zero -- invisible after abs and
// rint.
template <typename E, bool kExact = true, typename P>
__device__ __forceinline__ void bfly4(P& a, P& b, P& c, P& d) {
  const P s = E::add(a, b);
  const P t = E::sub(a, b);
  const P o0 = E::sub(E::add(s, c), d);
  const P o1 = E::add(E::sub(s, c), d);
  const P o2 = E::add(E::add(t, c), d);
  P o3;
  if constexpr (kExact) {
    const P u = E::sub(b, a);  // == (-a) + b, including the sign of zero
    o3 = E::add(E::add(u, c), d);
  } else {
    o3 = E::add(E::sub(c, t), d);
  }
  a = o0;
  b = o1;
  c = o2;
  d = o3;
}

// 16-byte chunk at swizzled word index s (a multiple of 4).
template <typename P>
__device__ __forceinline__ void st_chunk(P* sm, int s, const P& v0, const P& v1, const P& v2, const P& v3) {
  P* dst = sm + s;
  if constexpr (sizeof(P) == 4) {
    uint4 u;
    u.x = *reinterpret_cast<const uint32_t*>(&v0);
    u.y = *reinterpret_cast<const uint32_t*>(&v1);
    u.z = *reinterpret_cast<const uint32_t*>(&v2);
    u.w = *reinterpret_cast<const uint32_t*>(&v3);
    *reinterpret_cast<uint4*>(dst) = u;
  } else {
    dst[0] = v0;
    dst[1] = v1;
    dst[2] = v2;
    dst[3] = v3;
  }
}

template <typename P>
__device__ __forceinline__ void ld_chunk(const P* sm, int s, P& v0, P& v1, P& v2, P& v3) {
  const P* src = sm + s;
  if constexpr (sizeof(P) == 4) {
    const uint4 u = *reinterpret_cast<const uint4*>(src);
    v0 = *reinterpret_cast<const P*>(&u.x);
    v1 = *reinterpret_cast<const P*>(&u.y);
    v2 = *reinterpret_cast<const P*>(&u.z);
    v3 = *reinterpret_cast<const P*>(&u.w);
  } else {
    v0 = src[0];
    v1 = src[1];
    v2 = src[2];
    v3 = src[3];
  }
}

// Raw 16-element half-units as loaded from global memory.
template <typename T> struct Raw16 {
  static constexpr int kVec = 16 * sizeof(T) / 16;  // uint4 per 16 elements
  uint4 v[kVec];
};

template <typename T>
__device__ __forceinline__ void load16(Raw16<T>& r, const T* src) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int i = 0; i < Raw16<T>::kVec; ++i) r.v[i] = __ldg(s + i);
}

template <typename T>
__device__ __forceinline__ void load16_shared(Raw16<T>& r, const T* src) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int i = 0; i < Raw16<T>::kVec; ++i) r.v[i] = s[i];
}

template <typename T>
__device__ __forceinline__ void zero16(Raw16<T>& r) {
#pragma unroll
  for (int i = 0; i < Raw16<T>::kVec; ++i) r.v[i] = make_uint4(0, 0, 0, 0);
}

template <typename T>
__device__ __forceinline__ T raw_elem(const Raw16<T>& r, int i) {
  return reinterpret_cast<const T*>(r.v)[i];
}

template <typename E, typename T, typename P>
__device__ __forceinline__ void interleave(P (&v)[16], const Raw16<T>& lo, const Raw16<T>& hi) {
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = E::make(raw_elem(lo, i), raw_elem(hi, i));
}

// Radix-4 stages with strides 1 and 4 over 16 registers (stride 1 only for G == 4).
template <typename E, int G, bool kExact, typename P>
__device__ __forceinline__ void stages_1_4(P (&v)[16]) {
  if constexpr (G >= 4) {
#pragma unroll
    for (int j = 0; j < 4; ++j) bfly4<E, kExact>(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
  if constexpr (G >= 16) {
#pragma unroll
    for (int j = 0; j < 4; ++j) bfly4<E, kExact>(v[j], v[j + 4], v[j + 8], v[j + 12]);
  }
}

// bf16 quantizing modes skip the explicit x / sqrt(G) (a power of two: exact
// unless the value underflows, and then its code is 0 either way) and fold it
// into the reciprocal scale; the row absmax runs on packed bf16x2 words.
template <typename T, int MODE>
constexpr bool kFastQuant = std::is_same<T, __nv_bfloat16>::value && MODE != kModeRotate;

__device__ __forceinline__ void absmax_bf16x2(const __nv_bfloat162 (&v)[16], __nv_bfloat162& m) {
#pragma unroll
  for (int i = 0; i < 16; ++i) m = __hmax2(m, __habs2(v[i]));
}

template <typename E, typename P>
__device__ __forceinline__ float normalize_absmax(P (&v)[16], P nrm, float amax) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    v[i] = E::mul(v[i], nrm);
    amax = fmaxf(amax, fmaxf(fabsf(E::to_f(E::lo(v[i]))), fabsf(E::to_f(E::hi(v[i])))));
  }
  return amax;
}

template <typename E, typename T>
__device__ __forceinline__ int code_of(T v, float scale) {
  const float ratio = E::to_f(E::from_f(__fdiv_rn(E::to_f(v), scale)));
  const int q = __float2int_rn(ratio);  // half to even; NaN -> 0
  return min(max(q, -7), 7);
}

// Write 16 outputs of one half-unit.
template <typename E, typename T, int MODE>
__device__ __forceinline__ void write_half(void* out, int64_t row, int64_t K, int64_t col, const T (&e)[16],
                                           float scale) {
  if constexpr (MODE == kModeI8) {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t acc = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) acc |= (static_cast<uint32_t>(code_of<E>(e[4 * j + b], scale)) & 0xFFu) << (8 * b);
      w[j] = acc;
    }
    int8_t* o = static_cast<int8_t*>(out) + row * K + col;
    *reinterpret_cast<uint4*>(o) = make_uint4(w[0], w[1], w[2], w[3]);
  } else if constexpr (MODE == kModePacked) {
    uint32_t w[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint32_t acc = 0;
#pragma unroll
      for (int b = 0; b < 8; ++b) acc |= (static_cast<uint32_t>(code_of<E>(e[8 * j + b], scale)) & 0xFu) << (4 * b);
      w[j] = acc;
    }
    uint8_t* o = static_cast<uint8_t*>(out) + row * (K / 2) + col / 2;
    *reinterpret_cast<uint2*>(o) = make_uint2(w[0], w[1]);
  } else {
    T* o = static_cast<T*>(out) + row * K + col;
    const uint4* s = reinterpret_cast<const uint4*>(e);
    uint4* d = reinterpret_cast<uint4*>(o);
#pragma unroll
    for (int i = 0; i < Raw16<T>::kVec; ++i) d[i] = s[i];
  }
}

// bf16 codes of two elements.  With r = fl(1 / scale) (times the exact
// 2^-k normalization), RNE_bf16(fl(x * r)) == RNE_bf16(x / scale) for bf16 x
// and scale: a quotient of 8-bit significands is never a bf16 midpoint (its
// odd part would need >= 9 bits) and lies >= 2^-17 (relative) from every
// midpoint, while fl(x * r) is within 2^-23 of it.  Adding 136 in bf16 (ulp 1
// on [128, 256)) then rounds half-to-even to an integer and leaves 8 + code
// (code in [-7, 7]) in the low byte of each half.
__device__ __forceinline__ uint32_t codes2_bf16(__nv_bfloat162 v, float r) {
  const uint32_t bits = *reinterpret_cast<const uint32_t*>(&v);
  const float x0 = __uint_as_float(bits << 16);
  const float x1 = __uint_as_float(bits & 0xFFFF0000u);
  const float2 xr = mul2_rn(make_float2(x0, x1), make_float2(r, r));  // paired, rounded as __fmul_rn
  const __nv_bfloat162 q = __floats2bfloat162_rn(xr.x, xr.y);
  const __nv_bfloat162 t = __hadd2(q, __float2bfloat162_rn(136.0f));
  return *reinterpret_cast<const uint32_t*>(&t);
}

template <int MODE>
__device__ __forceinline__ void emit_unit_bf16(void* out, int64_t row, int64_t K, int half, int p0,
                                               const __nv_bfloat162 (&v)[16], float r) {
  uint32_t lo[4], hi[4];  // biased codes 8 + c, one per byte, elements p0.. and p0 + half..
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t t0 = codes2_bf16(v[4 * j], r), t1 = codes2_bf16(v[4 * j + 1], r);
    const uint32_t t2 = codes2_bf16(v[4 * j + 2], r), t3 = codes2_bf16(v[4 * j + 3], r);
    const uint32_t x = __byte_perm(t0, t1, 0x6240);  // lo0 lo1 hi0 hi1
    const uint32_t y = __byte_perm(t2, t3, 0x6240);
    lo[j] = __byte_perm(x, y, 0x5410);
    hi[j] = __byte_perm(x, y, 0x7632);
  }
  const bool hi_ok = p0 + half < K;
  if constexpr (MODE == kModeI8) {
    // byte 8 + c -> two's-complement c: (u + 0x78) ^ 0x80, no carry across bytes
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      lo[j] = (lo[j] + 0x78787878u) ^ 0x80808080u;
      hi[j] = (hi[j] + 0x78787878u) ^ 0x80808080u;
    }
    int8_t* o = static_cast<int8_t*>(out) + row * K;
    *reinterpret_cast<uint4*>(o + p0) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    if (hi_ok) *reinterpret_cast<uint4*>(o + p0 + half) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  } else {
    // nibble = (8 + c) ^ 8; two nibbles per byte, element 2j low
    uint32_t pl[2], ph[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint32_t a0 = lo[2 * j] ^ 0x08080808u, a1 = lo[2 * j + 1] ^ 0x08080808u;
      const uint32_t b0 = hi[2 * j] ^ 0x08080808u, b1 = hi[2 * j + 1] ^ 0x08080808u;
      pl[j] = __byte_perm((a0 | (a0 >> 4)) & 0x00FF00FFu, (a1 | (a1 >> 4)) & 0x00FF00FFu, 0x6420);
      ph[j] = __byte_perm((b0 | (b0 >> 4)) & 0x00FF00FFu, (b1 | (b1 >> 4)) & 0x00FF00FFu, 0x6420);
    }
    uint8_t* o = static_cast<uint8_t*>(out) + row * (K / 2);
    *reinterpret_cast<uint2*>(o + p0 / 2) = make_uint2(pl[0], pl[1]);
    if (hi_ok) *reinterpret_cast<uint2*>(o + (p0 + half) / 2) = make_uint2(ph[0], ph[1]);
  }
}

template <typename E, typename T, int MODE, typename P>
__device__ __forceinline__ void emit_unit(void* out, int64_t row, int64_t K, int half, int p0, const P (&v)[16],
                                          float scale) {
  T lo[16], hi[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    lo[i] = E::lo(v[i]);
    hi[i] = E::hi(v[i]);
  }
  write_half<E, T, MODE>(out, row, K, p0, lo, scale);
  if (p0 + half < K) write_half<E, T, MODE>(out, row, K, p0 + half, hi, scale);
}

// STAGED: the grid is persistent (as many CTAs as are resident; a CTA takes
// rows blockIdx.x, + gridDim.x, ...) and each row arrives in shared memory by
// one bulk copy, issued by thread 0 as soon as every thread has read the
// previous row's raw words (right after the row's one CTA barrier), so the
// copy overlaps the rest of the row.  The raw words then cost no registers:
// about twice the rows per SM are in flight than when every thread holds its
// raw words in registers (the unstaged form, for rows too long to stage).
// MINB > 1: the register cap of __launch_bounds__(256, MINB), which lets
// more of the small (one-unit-per-thread) CTAs share an SM; used where there
// are enough rows to fill them (measured on B200: 4096 x 3072 rows 8% faster
// at MINB 5, 1536 x 3072 rows 4% slower).
template <typename T, int G, int MODE, int UPT, bool STAGED, int MINB = 1>
__global__ void __launch_bounds__(256, MINB) prep_kernel(const T* __restrict__ x, int64_t rows, int K, int half,
                                                     void* __restrict__ out, float* __restrict__ scales,
                                                     int* __restrict__ err) {
  using E = Elem<T>;
  using P = typename E::Pair;
  constexpr bool kSmem = G >= 64;  // later stages need other threads' words
  extern __shared__ __align__(128) unsigned char smem_raw[];
  P* sm = reinterpret_cast<P*>(smem_raw);
  // raw row (STAGED) after the pair-words; half * sizeof(P) is a multiple of 64
  T* raw = reinterpret_cast<T*>(smem_raw + (kSmem ? static_cast<size_t>(half) * sizeof(P) : 0));
  __shared__ float red[2][32];  // per-warp maxima, double-buffered by row parity
  __shared__ __align__(8) uint64_t raw_full;
  __shared__ int abort_flag;

  const int tid = threadIdx.x;
  const int nthr = blockDim.x;
  const int units = half >> 4;
  constexpr float kNorm = G == 1 ? 1.0f : G == 4 ? 0.5f : G == 16 ? 0.25f : G == 64 ? 0.125f : G == 256 ? 0.0625f : 0.03125f;
  constexpr bool kFast = kFastQuant<T, MODE>;
  constexpr bool kExact = !kFast;
  const P nrm = E::splat(kNorm);

  // swizzled bases of this thread's accesses, the same for every row
  int s_unit[UPT], s_col[UPT], s_col3[UPT];
#pragma unroll
  for (int j = 0; j < UPT; ++j) {
    const int t = tid + j * nthr;
    s_unit[j] = swz(t << 4);                                // phase 1 and quantize: ^ swz(4m)
    s_col[j] = G == 64 ? swz(64 * (t >> 2) + 4 * (t & 3))   // phase 2, G = 64: ^ swz(16i)
                       : swz(256 * (t >> 4) + (t & 15));    // phase 2, G >= 256: ^ swz(16i)
    s_col3[j] = swz(1024 * (t >> 6) + ((t & 63) << 2));     // phase 3: ^ swz(256i)
  }
  const uint32_t row_bytes = static_cast<uint32_t>(K) * sizeof(T);
  if constexpr (STAGED) {
    if (tid == 0) {
      mbar_init(&raw_full, 1);
      abort_flag = 0;
      fence_mbar_init();
    }
    __syncthreads();
  }
  grid_dependency_wait();  // the input may come from the previous kernel of the stream
  grid_dependents_launch();
  if constexpr (STAGED) {
    if (tid == 0 && static_cast<int64_t>(blockIdx.x) < rows) {
      mbar_arrive_expect_tx(&raw_full, row_bytes);
      bulk_load_1d(raw, x + static_cast<int64_t>(blockIdx.x) * K, row_bytes, &raw_full);
    }
  }

  uint32_t iter = 0;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x, ++iter) {
    const T* xr = x + row * static_cast<int64_t>(K);
    if constexpr (STAGED) {
      // Bounded wait for this row's copy (1 s).  On time-out the flag is
      // raised and the CTA runs its remaining rows through every barrier
      // without copies or stores, so no thread is left waiting.
      if (!abort_flag) {
        const uint64_t t0 = globaltimer();
        for (uint32_t i = 0;; ++i) {
          if (mbar_try_wait(&raw_full, iter & 1)) break;
          if ((i & 255) == 255) {
            if (*reinterpret_cast<volatile int*>(&abort_flag)) break;
            if (globaltimer() - t0 > 1000000000ull) {
              atomicExch(&abort_flag, 1);
              break;
            }
          }
        }
      }
    }
    float amax = 0.0f;
    P amax2 = E::splat(0.0f);  // fast path: packed running max of |x|
    // last-stage bookkeeping: normalize + absmax (generic) or packed absmax (fast)
    auto finish = [&](P (&w)[16]) {
      if constexpr (kFast) {
        absmax_bf16x2(w, amax2);
      } else if constexpr (G > 1) {
        amax = normalize_absmax<E>(w, nrm, amax);
      } else {
        amax = normalize_absmax<E>(w, E::splat(1.0f), amax);
      }
    };

    // phase 1: unstaged, every global load of this thread first, then
    // rotate; staged, each unit's raw words come from shared memory just
    // before it is rotated (few registers live at a time).
    Raw16<T> rlo[UPT], rhi[UPT];
    if constexpr (!STAGED) {
#pragma unroll
      for (int j = 0; j < UPT; ++j) {
        const int u = tid + j * nthr;
        if (u < units) {
          const int p0 = u << 4;
          load16(rlo[j], xr + p0);
          if (p0 + half < K) load16(rhi[j], xr + p0 + half);
          else zero16(rhi[j]);
        }
      }
    }
    P v[UPT][16];
#pragma unroll
    for (int j = 0; j < UPT; ++j) {
      const int u = tid + j * nthr;
      if (u < units) {
        if constexpr (STAGED) {
          const int p0 = u << 4;
          load16_shared(rlo[j], raw + p0);
          if (p0 + half < K) load16_shared(rhi[j], raw + p0 + half);
          else zero16(rhi[j]);
        }
        interleave<E>(v[j], rlo[j], rhi[j]);
        stages_1_4<E, G, kExact>(v[j]);
        if constexpr (!kSmem) {
          finish(v[j]);
        } else {
          const int p0 = u << 4;
#pragma unroll
          for (int m = 0; m < 4; ++m) st_chunk(sm, s_unit[j] ^ swz(4 * m), v[j][4 * m], v[j][4 * m + 1], v[j][4 * m + 2], v[j][4 * m + 3]);
        }
      }
    }

    if constexpr (kSmem) {
      // Phase 2 works within blocks of 64 (G = 64) or 256 pair-words, whose
      // units and column tasks both belong to one quarter- or half-warp (task
      // and unit indices coincide, and the thread count is a multiple of 32),
      // so a warp barrier orders phase 1's stores before phase 2's loads.
      __syncwarp();
      // phase 2
#pragma unroll
      for (int j = 0; j < UPT; ++j) {
        const int t = tid + j * nthr;
        if (t >= units) continue;
        P w[16];
        if constexpr (G == 64) {
#pragma unroll
          for (int i = 0; i < 4; ++i) ld_chunk(sm, s_col[j] ^ swz(16 * i), w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
#pragma unroll
          for (int c = 0; c < 4; ++c) bfly4<E, kExact>(w[c], w[4 + c], w[8 + c], w[12 + c]);
          finish(w);
#pragma unroll
          for (int i = 0; i < 4; ++i) st_chunk(sm, s_col[j] ^ swz(16 * i), w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) w[i] = sm[s_col[j] ^ swz(16 * i)];
          stages_1_4<E, 16, kExact>(w);
          if constexpr (G == 256) finish(w);
#pragma unroll
          for (int i = 0; i < 16; ++i) sm[s_col[j] ^ swz(16 * i)] = w[i];
        }
      }
      if constexpr (G == 1024) {
        __syncthreads();
#pragma unroll
        for (int j = 0; j < UPT; ++j) {
          const int t = tid + j * nthr;
          if (t >= units) continue;
          P w[16];
#pragma unroll
          for (int i = 0; i < 4; ++i) ld_chunk(sm, s_col3[j] ^ swz(256 * i), w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
#pragma unroll
          for (int c = 0; c < 4; ++c) bfly4<E, kExact>(w[c], w[4 + c], w[8 + c], w[12 + c]);
          finish(w);
#pragma unroll
          for (int i = 0; i < 4; ++i) st_chunk(sm, s_col3[j] ^ swz(256 * i), w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
    }

    float scale = 1.0f, rscale = 1.0f;
    if constexpr (MODE != kModeRotate) {
      if constexpr (kFast) {
        // |x| of the unnormalized rotation; x / sqrt(G) is an exact power-of-two scale
        amax = fmaxf(__low2float(amax2), __high2float(amax2)) * kNorm;
      }
      // row absmax: warp shuffle, one barrier, then every warp reduces the
      // per-warp maxima itself
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
      if ((tid & 31) == 0) red[iter & 1][tid >> 5] = amax;
      __syncthreads();
      float rmax = (tid & 31) < (nthr >> 5) ? red[iter & 1][tid & 31] : 0.0f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) rmax = fmaxf(rmax, __shfl_xor_sync(0xFFFFFFFFu, rmax, o));
      const float floor_v = E::to_f(E::from_f(1.0e-10f));
      const float maximum = E::to_f(E::from_f(fmaxf(rmax, floor_v)));
      scale = E::to_f(E::from_f(__fdiv_rn(maximum, 7.0f)));
      rscale = __fdiv_rn(1.0f, scale) * kNorm;
    } else if constexpr (kSmem || STAGED) {
      __syncthreads();
    }
    if constexpr (STAGED) {
      // Every thread has read this row's raw words (they are in registers or
      // in the pair-word buffer): refill the raw buffer with the next row.
      // The proxy fence orders those generic reads before the copy's writes.
      if (tid == 0 && !abort_flag && row + gridDim.x < rows) {
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&raw_full, row_bytes);
        bulk_load_1d(raw, x + (row + gridDim.x) * static_cast<int64_t>(K), row_bytes, &raw_full);
      }
      if (abort_flag) continue;  // uniform: raised before the barrier above
    }
    if constexpr (MODE != kModeRotate) {
      if (tid == 0) scales[row] = scale;
    }

    // quantize (or emit the rotation)
#pragma unroll
    for (int j = 0; j < UPT; ++j) {
      const int u = tid + j * nthr;
      if (u >= units) continue;
      const int p0 = u << 4;
      if constexpr (kSmem) {
        P w[16];
#pragma unroll
        for (int m = 0; m < 4; ++m) ld_chunk(sm, s_unit[j] ^ swz(4 * m), w[4 * m], w[4 * m + 1], w[4 * m + 2], w[4 * m + 3]);
        if constexpr (kFast) emit_unit_bf16<MODE>(out, row, K, half, p0, w, rscale);
        else emit_unit<E, T, MODE>(out, row, K, half, p0, w, scale);
      } else {
        if constexpr (kFast) emit_unit_bf16<MODE>(out, row, K, half, p0, v[j], rscale);
        else emit_unit<E, T, MODE>(out, row, K, half, p0, v[j], scale);
      }
    }
    // Reuse by the next row: the raw buffer is refilled only after the next
    // CTA barrier above; `red` alternates by row parity; the pair-words of a
    // unit are rewritten by the same quarter- or half-warp that reads them
    // (ordered by warp barriers), and for G = 1024 only after the next row's
    // CTA barrier before phase 3.
    if constexpr (!STAGED) {
      if (row + gridDim.x < rows) __syncthreads();
    }
  }
  if constexpr (STAGED) {
    if (tid == 0 && abort_flag) {
      atomicCAS(err, 0, 41);
      const uint64_t t0 = globaltimer();  // let a copy still in flight land
      while (globaltimer() - t0 < 2000000ull) {
      }
    }
  }
}

// ---------------------------------------------------------------------------
// host dispatch

constexpr int64_t kPrepManyRows = 2048;  // rows from which the MINB = 5 form is used

template <typename T, int G, int MODE>
static int launch_g(const void* x, int64_t rows, int K, int half, void* out, float* scales, cudaStream_t stream) {
  const int units = half / 16;
  int upt = 1;
  while (upt < 8 && (units + upt - 1) / upt > 256) upt *= 2;
  int threads = ((units + upt - 1) / upt + 31) / 32 * 32;
  CONVROT_REQUIRE(threads <= 256, CONVROT_ERR_UNSUPPORTED, "features %d too large for the fused kernel", K);
  using P = typename Elem<T>::Pair;
  const size_t pair_bytes = G >= 64 ? static_cast<size_t>(half) * sizeof(P) : 0;
  CONVROT_REQUIRE(pair_bytes <= 227 * 1024, CONVROT_ERR_UNSUPPORTED, "features %d too large for the fused kernel", K);
  if (rows == 0) return CONVROT_OK;
  // Stage rows of 16 KB and more through shared memory (shorter rows fit
  // enough CTAs per SM unstaged), while pair-words + raw row leave room for at
  // least two CTAs per SM.
  const size_t row_bytes = static_cast<size_t>(K) * sizeof(T);
  const size_t staged_bytes = pair_bytes + row_bytes;
  const bool staged = row_bytes >= 16 * 1024 && staged_bytes <= 100 * 1024;
  const size_t smem = staged ? staged_bytes : pair_bytes;
  int* err = device_error_word();
  CONVROT_REQUIRE(err != nullptr, CONVROT_ERR_CUDA, "device error word unavailable");
  auto run = [&](auto kernel) -> int {
    CONVROT_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    int64_t grid_rows = rows < 2147483647LL ? rows : 2147483647LL;
    if (staged) {  // persistent: as many CTAs as are resident at once
      int per_sm = 0;
      CONVROT_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem));
      const int64_t resident = static_cast<int64_t>(per_sm > 0 ? per_sm : 1) * device_sm_count();
      if (resident < grid_rows) grid_rows = resident;
    }
    const unsigned grid = static_cast<unsigned>(grid_rows);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(static_cast<unsigned>(threads), 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see grid_dependency_wait
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CONVROT_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, static_cast<const T*>(x), rows, K, half, out, scales, err));
    return check_launch("convrot prep kernel");
  };
  if (staged) {
    switch (upt) {
      case 1: return run(prep_kernel<T, G, MODE, 1, true>);
      case 2: return run(prep_kernel<T, G, MODE, 2, true>);
      case 4: return run(prep_kernel<T, G, MODE, 4, true>);
      default: return run(prep_kernel<T, G, MODE, 8, true>);
    }
  }
  if (upt == 1 && rows >= kPrepManyRows) return run(prep_kernel<T, G, MODE, 1, false, 5>);
  switch (upt) {
    case 1: return run(prep_kernel<T, G, MODE, 1, false>);
    case 2: return run(prep_kernel<T, G, MODE, 2, false>);
    case 4: return run(prep_kernel<T, G, MODE, 4, false>);
    default: return run(prep_kernel<T, G, MODE, 8, false>);
  }
}

template <typename T, int MODE>
int launch_t(const void* x, int64_t rows, int64_t K, int G, void* out, float* scales, cudaStream_t stream) {
  const int64_t groups = K / G;
  const int64_t half = G == 1 ? K / 2 : ((groups + 1) / 2) * G;
  CONVROT_REQUIRE(half % 16 == 0, CONVROT_ERR_UNSUPPORTED,
                  "features %lld with group %d: the fused kernel needs half-rows of a multiple of 16 elements",
                  static_cast<long long>(K), G);
  CONVROT_REQUIRE(K <= (1 << 30), CONVROT_ERR_UNSUPPORTED, "features too large");
  const int k = static_cast<int>(K), h = static_cast<int>(half);
  switch (G) {
    case 1: return launch_g<T, 1, MODE>(x, rows, k, h, out, scales, stream);
    case 4: return launch_g<T, 4, MODE>(x, rows, k, h, out, scales, stream);
    case 16: return launch_g<T, 16, MODE>(x, rows, k, h, out, scales, stream);
    case 64: return launch_g<T, 64, MODE>(x, rows, k, h, out, scales, stream);
    case 256: return launch_g<T, 256, MODE>(x, rows, k, h, out, scales, stream);
    case 1024: return launch_g<T, 1024, MODE>(x, rows, k, h, out, scales, stream);
    default: break;
  }
  set_error("group size %d is not supported (supported: 1, 4, 16, 64, 256, 1024)", G);
  return CONVROT_ERR_UNSUPPORTED;
}

// Explicit instantiations live in prep_bf16.cu / prep_f16.cu / prep_f32.cu so
// the three dtypes compile in parallel.
#define CONVROT_PREP_INSTANTIATE(T)                                                                          \
  template int launch_t<T, kModeI8>(const void*, int64_t, int64_t, int, void*, float*, cudaStream_t);     \
  template int launch_t<T, kModePacked>(const void*, int64_t, int64_t, int, void*, float*, cudaStream_t); \
  template int launch_t<T, kModeRotate>(const void*, int64_t, int64_t, int, void*, float*, cudaStream_t);

}  // namespace convrot
