// Gather + dequantise of a 4-bit weight whose flat storage is split over the
// ranks of one node, read straight from the owners' memory (CUDA IPC pointers,
// plain 16-byte loads over NVLink; never TMA).
//
// The weight W [N, K] is stored in the bitsandbytes layout: row-major codes,
// two per byte (element 2i in the high nibble), one fp32 absmax per block of
// `blocksize` consecutive elements.  Rank q holds packed bytes
// [pstart[q], pstart[q+1]) and absmax entries [astart[q], astart[q+1]) of the
// flat arrays (uniform or weighted plans alike: the starts are the plan's
// offsets, the last entry is the total).  The reference assembles the same
// flat arrays with two all-gathers and unpad copies before dequantising
// (src/coordinator.py:385-533, src/hetero/zeroq_hetero.py:312-452).
//
// A gather item is 8 rows x 1024 columns of W, handled by one warp: lane l
// owns 32 consecutive columns (16 packed bytes, inside one absmax block when
// blocksize % 32 == 0) of each of the 8 rows, issues all 8 row loads before
// decoding any, and writes 8 x 64 contiguous bytes of bf16.
//
// The same machinery gathers fp32 master weights split over the ranks (the
// train-from-scratch layout: rank q holds flat elements [pstart[q],
// pstart[q+1]), reference src/coordinator.py:606-611 all-gathers them) and
// casts them to bf16: items of 8 rows x 256 columns, 8 consecutive fp32 per
// lane and row (two 16-byte loads), one 16-byte bf16 store.
#pragma once

#include "common.cuh"

namespace zq {

constexpr int kAgMaxRanks = 8;
constexpr int kAgRows = 8;          // rows of W per gather item
constexpr int kAgCols = 1024;       // columns of W per 4-bit gather item (32 per lane)
constexpr int kAgColsF32 = 256;     // columns of W per fp32 gather item (8 per lane)

enum AgKind { kAgNf4 = 0, kAgF32 = 1 };

struct AgSource {
  const uint8_t* packed[kAgMaxRanks];  // kAgF32: the fp32 pieces
  const float* absmax[kAgMaxRanks];
  int64_t pstart[kAgMaxRanks + 1];  // pstart[world] = total packed bytes (kAgF32: elements)
  int64_t astart[kAgMaxRanks + 1];  // astart[world] = total absmax entries
  int world;
  int kind;                         // AgKind
};

// Piece of flat index idx: the last rank whose start is <= idx (ranks with an
// empty piece share their start with the next rank and are skipped).  Written
// as a select chain over static indices so the table stays in the parameter
// bank (a dynamic index would copy it to the stack).
struct AgPiece {
  const void* base;
  int64_t start, end;
};

__device__ __forceinline__ AgPiece ag_packed_piece(const AgSource& s, int64_t idx) {
  AgPiece p{s.packed[0], s.pstart[0], s.pstart[1]};
#pragma unroll
  for (int r = 1; r < kAgMaxRanks; ++r)
    if (r < s.world && idx >= s.pstart[r]) p = AgPiece{s.packed[r], s.pstart[r], s.pstart[r + 1]};
  return p;
}

__device__ __forceinline__ AgPiece ag_absmax_piece(const AgSource& s, int64_t idx) {
  AgPiece p{s.absmax[0], s.astart[0], s.astart[1]};
#pragma unroll
  for (int r = 1; r < kAgMaxRanks; ++r)
    if (r < s.world && idx >= s.astart[r]) p = AgPiece{s.absmax[r], s.astart[r], s.astart[r + 1]};
  return p;
}

__device__ __forceinline__ uint4 ld_v4_no_l1(const void* p) {
  uint4 v;
  asm volatile("ld.global.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// 16 packed bytes starting at flat byte b, byte by byte (a piece boundary or an
// unaligned piece base falls inside them).
__device__ __forceinline__ uint4 ag_load16_bytes(const AgSource& s, int64_t b) {
  uint32_t w[4] = {0u, 0u, 0u, 0u};
  for (int i = 0; i < 16; ++i) {
    const AgPiece p = ag_packed_piece(s, b + i);
    w[i >> 2] |= (uint32_t)reinterpret_cast<const uint8_t*>(p.base)[b + i - p.start] << (8 * (i & 3));
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// fp32 code value x absmax, rounded once to bf16, for 32 codes (16 bytes);
// the same arithmetic as the standalone dequantise kernels.
__device__ __forceinline__ void ag_decode_store32(const uint4& raw, float am, const float* lut,
                                                  uint4* dst) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t byte = (w[i] >> (8 * q)) & 0xFFu;
      o[q] = pack_bf16x2(lut[byte >> 4] * am, lut[byte & 15u] * am);
    }
    dst[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Rows [r0, r0 + 8) x columns [k0, k0 + 1024) of W (clipped to N and K) into
// w_out [N, K] bf16.  Needs K % 32 == 0 and blocksize % 32 == 0.  The pieces
// holding the item's first packed byte and first absmax entry are looked up
// once; when they hold the whole item (the usual case: pieces are large) every
// lane indexes them directly, otherwise each row is resolved on its own.
__device__ __forceinline__ void ag_item(const AgSource& s, const float* lut, int N, int K,
                                        int blocksize, int r0, int k0, __nv_bfloat16* w_out,
                                        int lane) {
  const int rows_here = min(kAgRows, N - r0);
  const int cols_here = min(kAgCols, K - k0);
  const int64_t e_first = (int64_t)r0 * K + k0;
  const int64_t e_end = (int64_t)(r0 + rows_here - 1) * K + k0 + cols_here;  // exclusive
  const AgPiece pp = ag_packed_piece(s, e_first >> 1);
  const AgPiece pa = ag_absmax_piece(s, e_first / blocksize);
  const bool fast = (e_end >> 1) <= pp.end && (e_end - 1) / blocksize < pa.end &&
                    ((reinterpret_cast<uintptr_t>(pp.base) - (uintptr_t)pp.start) & 15) == 0;
  const int k = k0 + lane * 32;
  if (k >= K) return;
  if (!fast) {
#pragma unroll 1
    for (int i = 0; i < rows_here; ++i) {
      const int64_t e = (int64_t)(r0 + i) * K + k;
      const int64_t ai = e / blocksize;
      const AgPiece q = ag_absmax_piece(s, ai);
      ag_decode_store32(ag_load16_bytes(s, e >> 1), reinterpret_cast<const float*>(q.base)[ai - q.start],
                        lut, reinterpret_cast<uint4*>(w_out + (int64_t)(r0 + i) * K + k));
    }
    return;
  }
  // indexed by the flat (global) byte / block number
  const uint8_t* pbase = reinterpret_cast<const uint8_t*>(pp.base) - pp.start;
  const float* abase = reinterpret_cast<const float*>(pa.base) - pa.start;
  uint4 raw[kAgRows];
  float am[kAgRows];
#pragma unroll
  for (int i = 0; i < kAgRows; ++i) {
    if (i < rows_here) {
      const int64_t e = (int64_t)(r0 + i) * K + k;
      raw[i] = ld_v4_no_l1(pbase + (e >> 1));
      am[i] = abase[e / blocksize];
    }
  }
#pragma unroll
  for (int i = 0; i < kAgRows; ++i) {
    if (i < rows_here)
      ag_decode_store32(raw[i], am[i], lut,
                        reinterpret_cast<uint4*>(w_out + (int64_t)(r0 + i) * K + k));
  }
}

// Rows [r0, r0 + 8) x columns [k0, k0 + 256) of the fp32 W (clipped to N and
// K) cast to bf16 into w_out [N, K].  Needs K % 8 == 0.
__device__ __forceinline__ void ag_item_f32(const AgSource& s, int N, int K, int r0, int k0,
                                            __nv_bfloat16* w_out, int lane) {
  const int rows_here = min(kAgRows, N - r0);
  const int cols_here = min(kAgColsF32, K - k0);
  const int64_t e_first = (int64_t)r0 * K + k0;
  const int64_t e_end = (int64_t)(r0 + rows_here - 1) * K + k0 + cols_here;  // exclusive
  const AgPiece pp = ag_packed_piece(s, e_first);
  const bool fast = e_end <= pp.end &&
                    ((reinterpret_cast<uintptr_t>(pp.base) - (uintptr_t)(pp.start * 4)) & 15) == 0;
  const int k = k0 + lane * 8;
  if (k >= K) return;
  if (!fast) {
#pragma unroll 1
    for (int i = 0; i < rows_here; ++i) {
      const int64_t e = (int64_t)(r0 + i) * K + k;
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const AgPiece a = ag_packed_piece(s, e + 2 * j);
        const AgPiece b = ag_packed_piece(s, e + 2 * j + 1);
        o[j] = pack_bf16x2(reinterpret_cast<const float*>(a.base)[e + 2 * j - a.start],
                           reinterpret_cast<const float*>(b.base)[e + 2 * j + 1 - b.start]);
      }
      *reinterpret_cast<uint4*>(w_out + (int64_t)(r0 + i) * K + k) = make_uint4(o[0], o[1], o[2], o[3]);
    }
    return;
  }
  const float* fbase = reinterpret_cast<const float*>(pp.base) - pp.start;
  // two passes of 4 rows: 8 loads (4 KB per warp) in flight per pass
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint4 lo[4], hi[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (half * 4 + i < rows_here) {
        const float* src = fbase + (int64_t)(r0 + half * 4 + i) * K + k;
        lo[i] = ld_v4_no_l1(src);
        hi[i] = ld_v4_no_l1(src + 4);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (half * 4 + i < rows_here) {
        const uint4 o = make_uint4(
            pack_bf16x2(__uint_as_float(lo[i].x), __uint_as_float(lo[i].y)),
            pack_bf16x2(__uint_as_float(lo[i].z), __uint_as_float(lo[i].w)),
            pack_bf16x2(__uint_as_float(hi[i].x), __uint_as_float(hi[i].y)),
            pack_bf16x2(__uint_as_float(hi[i].z), __uint_as_float(hi[i].w)));
        *reinterpret_cast<uint4*>(w_out + (int64_t)(r0 + half * 4 + i) * K + k) = o;
      }
    }
  }
}

}  // namespace zq
