// One layer's attention input in one pass, for sm_100a: per-head RMSNorm of Q
// and K, rotary embedding of Q and K, Q written out, K and V stored into the
// paged pool by slot.
//
// Work item = one chunk of G consecutive heads of one kind (Q, K or V) of one
// token, enumerated token-major over the token's Q chunks, then K, then V.
// One warp per chunk, two head rows at a time: half-warp h = lane / 16 takes
// row 2 pr + h of row pair pr, and lane l = lane % 16 holds elements
// [l Q, l Q + Q) ("low") and [D/2 + l Q, D/2 + l Q + Q) ("high") of that row,
// Q = head_dim / 32.  Both members of a neox pair (j, j + D/2) and of a GPT-J
// pair (2j, 2j + 1) then sit in the same lane, one 4-level shuffle reduction
// serves both rows' sums of squares, and the arithmetic runs on packed fp32
// pairs (FMUL2 / FFMA2), which round each component exactly as scalar fp32.
//
// Two kernels share that chunk arithmetic:
// * qkv_norm_rope_store_kernel: each warp loads its chunk's rows, the token's
//   slot, position, cos/sin row and the weights into registers before using
//   any of them.  One row pair per warp for small batches (decode), where
//   the whole batch is a single wave; 8-head chunks (4 at head_dim 256) for
//   large ones whose copies cannot use the TMA kernel.
// * qkv_tma_kernel: one CTA per SM; a producer warp streams tiles of whole
//   tokens (Q, K, V rows and the token's cos/sin row) into a ring of shared
//   memory stages with bulk copies completing on mbarriers, 16 consumer warps
//   take the chunks of a landed stage (6 stages of 2-3 tokens by default).
//   The bytes in flight live in shared memory (up to 227 KB per SM)
//   instead of registers, which is what HBM
//   latency x bandwidth asks for at prefill sizes.  Every mbarrier wait is
//   bounded; a timeout sets YL_DEVERR_TIMEOUT and the CTA drains its copies
//   and exits.
//
// Reference: flashinfer::norm::QKRMSNorm as called by RSMNormWithoutResidual
// (src/layers/rsm_norm.cu:35-52) computes out = x * rsqrt(sum(x^2) / d + eps)
// * w in fp32 per head; StoreKVCacheKernel (src/kvcache/store_kv_cache.cu:46-77)
// places K/V rows by slot.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <string>

#include "common.cuh"
#include "tma.cuh"

namespace ylk {

struct QkvParams {
  const char *q;
  const char *k;
  const char *v;
  char *q_out;
  char *k_cache;
  char *v_cache;
  const void *slots;
  const char *q_weight;
  const char *k_weight;
  const float *cos_sin;
  const void *positions;
  int64_t q_stride;
  int64_t k_stride;
  int64_t v_stride;
  int64_t q_out_stride;
  int64_t cache_stride;
  int64_t num_slots;
  int64_t max_position;
  uint32_t *error_word;
  uint32_t num_tokens;
  uint32_t items;   // register kernel: N * chunks  (< 2^31)
  uint32_t hq;
  uint32_t hk;
  uint32_t cq;      // chunks of G Q heads per token
  uint32_t ck;      // chunks of G K (and of V) heads per token
  uint32_t chunks;  // cq + 2 ck
  FastDiv by_chunks;
  float eps;
  int slot64;
  int pos64;
  int interleaved;
  // TMA kernel: tiles of tile_tokens tokens, one stage each
  uint32_t tile_tokens;
  uint32_t num_tiles;
  uint32_t token_bytes;  // Q + K + V rows (+ cos/sin row) of one token in a stage
  uint32_t stage_bytes;  // meta + tile_tokens * token_bytes
  uint32_t num_stages;   // <= kQkvMaxStages
};

// 16-bit element types: a pair of elements is one 32-bit word, low half first.
template <typename T>
struct Elem;
template <>
struct Elem<__nv_bfloat16> {
  // bf16 -> fp32 is exact: the bf16 bits are the high half of the fp32 bits
  static __device__ __forceinline__ float lo(uint32_t w) { return __uint_as_float(w << 16); }
  static __device__ __forceinline__ float hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
  static __device__ __forceinline__ float2 pair(uint32_t w) { return make_float2(lo(w), hi(w)); }
  static __device__ __forceinline__ uint32_t pack(float a, float b) {  // round to nearest even
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
  }
};
template <>
struct Elem<__half> {
  static __device__ __forceinline__ float lo(uint32_t w) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xffffu)));
  }
  static __device__ __forceinline__ float hi(uint32_t w) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
  }
  static __device__ __forceinline__ float2 pair(uint32_t w) { return make_float2(lo(w), hi(w)); }
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
  }
};

// WORDS 32-bit words: 2 * WORDS 16-bit elements of one lane.
template <int WORDS>
struct Words {
  uint32_t w[WORDS];
};

// A packed fp32 pair rounded to one word of two 16-bit elements.
template <typename E>
__device__ __forceinline__ uint32_t pack2(float2 v) {
  return E::pack(v.x, v.y);
}

// Input rows are read once: non-coherent path, no L1 allocation.
template <int WORDS>
__device__ __forceinline__ void load_once(Words<WORDS> &x, const char *p) {
  if constexpr (WORDS == 1) {
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(x.w[0]) : "l"(p));
  } else if constexpr (WORDS == 2) {
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(x.w[0]), "=r"(x.w[1]) : "l"(p));
  } else {
    static_assert(WORDS == 4, "head_dim 64, 128 or 256");
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(x.w[0]), "=r"(x.w[1]), "=r"(x.w[2]), "=r"(x.w[3])
                 : "l"(p));
  }
}

// Weights (read by every row) and shared-memory rows: plain vector loads.
template <int WORDS>
__device__ __forceinline__ void load_words(Words<WORDS> &x, const char *p) {
  if constexpr (WORDS == 1) {
    x.w[0] = *reinterpret_cast<const uint32_t *>(p);
  } else if constexpr (WORDS == 2) {
    const uint2 t = *reinterpret_cast<const uint2 *>(p);
    x.w[0] = t.x, x.w[1] = t.y;
  } else {
    const uint4 t = *reinterpret_cast<const uint4 *>(p);
    x.w[0] = t.x, x.w[1] = t.y, x.w[2] = t.z, x.w[3] = t.w;
  }
}

template <int WORDS>
__device__ __forceinline__ void store_words(char *p, const Words<WORDS> &x) {
  if constexpr (WORDS == 1) {
    *reinterpret_cast<uint32_t *>(p) = x.w[0];
  } else if constexpr (WORDS == 2) {
    *reinterpret_cast<uint2 *>(p) = make_uint2(x.w[0], x.w[1]);
  } else {
    *reinterpret_cast<uint4 *>(p) = make_uint4(x.w[0], x.w[1], x.w[2], x.w[3]);
  }
}

// n consecutive fp32 values from a 4n-byte aligned address (n = 1, 2, 4, 8).
template <int N>
__device__ __forceinline__ void load_floats(float (&out)[N], const float *p) {
  if constexpr (N == 1) {
    out[0] = *p;
  } else if constexpr (N == 2) {
    const float2 t = *reinterpret_cast<const float2 *>(p);
    out[0] = t.x, out[1] = t.y;
  } else {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
      const float4 t = *reinterpret_cast<const float4 *>(p + i);
      out[i] = t.x, out[i + 1] = t.y, out[i + 2] = t.z, out[i + 3] = t.w;
    }
  }
}

template <typename IntT>
__device__ __forceinline__ int64_t load_int(const void *p, uint32_t i) {
  return static_cast<int64_t>(__ldg(static_cast<const IntT *>(p) + i));
}

// Lane geometry of a head row of D elements.
template <int D>
struct Lay {
  static constexpr int Q = D / 32;    // elements per segment
  static constexpr int W = Q / 2;     // 32-bit words per segment
  static constexpr int SEG = Q * 2;   // bytes per segment
  static constexpr int ROW = D * 2;   // bytes per row
  static constexpr int HALF = D;      // byte offset of the high segment
};

// Rotation coefficients of this lane for one token.  neox: c[i], s[i] are
// pair l Q + i, shared by element i of the low and of the high segment.
// GPT-J: c[k], s[k] (k < W) are the pair of low word k, c[W + k], s[W + k]
// the pair of high word k.
template <int D>
struct Rot {
  float c[Lay<D>::Q], s[Lay<D>::Q];
};

// From a cos/sin row (D/2 cosines, then D/2 sines).  GPT-J: low word k is
// pair l Q / 2 + k, high word k is pair D/4 + l Q / 2 + k.
template <int D>
__device__ __forceinline__ void load_rotation(Rot<D> &r, const float *row, uint32_t l, bool interleaved) {
  constexpr int Q = Lay<D>::Q, W = Lay<D>::W;
  if (!interleaved) {
    load_floats(r.c, row + l * Q);
    load_floats(r.s, row + D / 2 + l * Q);
  } else {
    float cl[W], ch[W], sl[W], sh[W];
    load_floats(cl, row + l * W);
    load_floats(ch, row + D / 4 + l * W);
    load_floats(sl, row + D / 2 + l * W);
    load_floats(sh, row + D / 2 + D / 4 + l * W);
#pragma unroll
    for (int k = 0; k < W; ++k) r.c[k] = cl[k], r.c[W + k] = ch[k], r.s[k] = sl[k], r.s[W + k] = sh[k];
  }
}

__device__ __forceinline__ float2 swap(float2 v) { return make_float2(v.y, v.x); }

// Norm, rotation and store of the PR row pairs of a chunk (Q or K rows):
// lo[pr] / hi[pr] hold this lane's segments of row 2 pr + lane / 16, rows
// g < nh are stored at dst + g * D * 2.
template <typename T, int D, int PR>
__device__ __forceinline__ void finish_pairs(const Words<Lay<D>::W> (&lo)[PR], const Words<Lay<D>::W> (&hi)[PR],
                                             uint32_t nh, const char *w, float eps, bool rope, bool interleaved,
                                             const Rot<D> &rot, uint32_t lane, char *dst) {
  using L = Lay<D>;
  constexpr int W = L::W;
  using E = Elem<T>;
  const uint32_t l = lane & 15u;
  float2 a[PR][W], b[PR][W];
#pragma unroll
  for (int pr = 0; pr < PR; ++pr)
#pragma unroll
    for (int k = 0; k < W; ++k) a[pr][k] = E::pair(lo[pr].w[k]), b[pr][k] = E::pair(hi[pr].w[k]);
  if (w != nullptr) {
    Words<W> wl, wh;
    load_words(wl, w + l * L::SEG);
    load_words(wh, w + L::HALF + l * L::SEG);
    float ss[PR];
#pragma unroll
    for (int pr = 0; pr < PR; ++pr) {
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int k = 0; k < W; ++k) {
        acc = __ffma2_rn(a[pr][k], a[pr][k], acc);
        acc = __ffma2_rn(b[pr][k], b[pr][k], acc);
      }
      ss[pr] = acc.x + acc.y;
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1)
#pragma unroll
      for (int pr = 0; pr < PR; ++pr) ss[pr] += __shfl_xor_sync(0xffffffffu, ss[pr], o);
#pragma unroll
    for (int pr = 0; pr < PR; ++pr) {
      const float r = rsqrtf(ss[pr] * (1.f / static_cast<float>(D)) + eps);  // 1/D is exact (D a power of 2)
      const float2 rr = make_float2(r, r);
#pragma unroll
      for (int k = 0; k < W; ++k) {
        // (x * r) * w, rounded to T: the norm's output is a T tensor in the unfused sequence
        a[pr][k] = E::pair(pack2<E>(__fmul2_rn(__fmul2_rn(a[pr][k], rr), E::pair(wl.w[k]))));
        b[pr][k] = E::pair(pack2<E>(__fmul2_rn(__fmul2_rn(b[pr][k], rr), E::pair(wh.w[k]))));
      }
    }
  }
  if (rope) {
    if (!interleaved) {
      // y_lo = a c - b s,  y_hi = b c + a s
#pragma unroll
      for (int k = 0; k < W; ++k) {
        const float2 c = make_float2(rot.c[2 * k], rot.c[2 * k + 1]);
        const float2 sn = make_float2(rot.s[2 * k], rot.s[2 * k + 1]);
        const float2 ns = make_float2(-rot.s[2 * k], -rot.s[2 * k + 1]);
#pragma unroll
        for (int pr = 0; pr < PR; ++pr) {
          const float2 ya = __ffma2_rn(a[pr][k], c, __fmul2_rn(b[pr][k], ns));
          const float2 yb = __ffma2_rn(b[pr][k], c, __fmul2_rn(a[pr][k], sn));
          a[pr][k] = ya, b[pr][k] = yb;
        }
      }
    } else {
      // (x0, x1) -> (x0 c - x1 s, x1 c + x0 s)
#pragma unroll
      for (int k = 0; k < W; ++k) {
        const float2 ml = make_float2(rot.c[k], rot.c[k]), pl = make_float2(-rot.s[k], rot.s[k]);
        const float2 mh = make_float2(rot.c[W + k], rot.c[W + k]), ph = make_float2(-rot.s[W + k], rot.s[W + k]);
#pragma unroll
        for (int pr = 0; pr < PR; ++pr) {
          a[pr][k] = __ffma2_rn(a[pr][k], ml, __fmul2_rn(swap(a[pr][k]), pl));
          b[pr][k] = __ffma2_rn(b[pr][k], mh, __fmul2_rn(swap(b[pr][k]), ph));
        }
      }
    }
  }
  const uint32_t half = lane >> 4;
  dst += l * L::SEG;
#pragma unroll
  for (int pr = 0; pr < PR; ++pr) {
    const uint32_t g = 2 * pr + half;
    if (g < nh) {
      Words<W> yl, yh;
#pragma unroll
      for (int k = 0; k < W; ++k) yl.w[k] = pack2<E>(a[pr][k]), yh.w[k] = pack2<E>(b[pr][k]);
      store_words(dst + g * L::ROW, yl);
      store_words(dst + g * L::ROW + L::HALF, yh);
    }
  }
}

// Copy of the PR row pairs of a V chunk to dst (rows g < nh).
template <int D, int PR>
__device__ __forceinline__ void copy_pairs(const Words<Lay<D>::W> (&lo)[PR], const Words<Lay<D>::W> (&hi)[PR],
                                           uint32_t nh, uint32_t lane, char *dst) {
  using L = Lay<D>;
  const uint32_t half = lane >> 4;
  dst += (lane & 15u) * L::SEG;
#pragma unroll
  for (int pr = 0; pr < PR; ++pr) {
    const uint32_t g = 2 * pr + half;
    if (g < nh) {
      store_words(dst + g * L::ROW, lo[pr]);
      store_words(dst + g * L::ROW + L::HALF, hi[pr]);
    }
  }
}

// Kind (0 Q, 1 K, 2 V), first head and head count of chunk c of a token.
__device__ __forceinline__ void chunk_heads(const QkvParams &p, uint32_t c, uint32_t G, int &kind, uint32_t &h0,
                                            uint32_t &nh) {
  kind = c < p.cq ? 0 : (c < p.cq + p.ck ? 1 : 2);
  h0 = (kind == 0 ? c : (kind == 1 ? c - p.cq : c - p.cq - p.ck)) * G;
  nh = min(G, (kind == 0 ? p.hq : p.hk) - h0);
}

// True when the token's K/V rows go to the pool; -1 skips silently.
__device__ __forceinline__ bool slot_ok(const QkvParams &p, int64_t slot, uint32_t lane) {
  const bool ok = slot >= 0 && (p.num_slots <= 0 || slot < p.num_slots);
  if (!ok && slot != -1 && lane == 0) raise_deverr(p.error_word, YL_DEVERR_SLOT_RANGE);
  return ok;
}

template <typename T, int D, int G>
__global__ void __launch_bounds__(256) qkv_norm_rope_store_kernel(const __grid_constant__ QkvParams p) {
  static_assert(G % 2 == 0, "row pairs");
  using L = Lay<D>;
  constexpr int PR = G / 2;
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint32_t num_warps = (gridDim.x * blockDim.x) >> 5;
  const uint32_t lane_off = (lane & 15u) * L::SEG + (lane >> 4) * L::ROW;  // this lane's low segment in a pair
  pdl_wait();  // Q/K/V may be written by the kernel just before this one
  for (uint32_t item = warp; item < p.items; item += num_warps) {
    const uint32_t tok = p.by_chunks.div(item);
    int kind;
    uint32_t h0, nh;
    chunk_heads(p, item - tok * p.chunks, G, kind, h0, nh);
    const char *src = (kind == 0 ? p.q + tok * p.q_stride : (kind == 1 ? p.k + tok * p.k_stride : p.v + tok * p.v_stride)) +
                      h0 * L::ROW + lane_off;
    // every load of the chunk before any use
    Words<L::W> lo[PR], hi[PR];
#pragma unroll
    for (int pr = 0; pr < PR; ++pr)
      if (2 * pr + (lane >> 4) < nh) {
        load_once(lo[pr], src + 2 * pr * L::ROW);
        load_once(hi[pr], src + 2 * pr * L::ROW + L::HALF);
      }
    int64_t slot = 0;
    if (kind != 0) slot = p.slot64 ? load_int<int64_t>(p.slots, tok) : load_int<int32_t>(p.slots, tok);
    int64_t pos = 0;
    if (p.cos_sin != nullptr) pos = p.pos64 ? load_int<int64_t>(p.positions, tok) : load_int<int32_t>(p.positions, tok);
    if (p.cos_sin != nullptr && (pos < 0 || pos >= p.max_position)) {
      if (lane == 0) raise_deverr(p.error_word, YL_DEVERR_POSITION_RANGE);
      continue;
    }
    if (kind != 0 && !slot_ok(p, slot, lane)) continue;
    if (kind == 2) {
      copy_pairs<D, PR>(lo, hi, nh, lane, p.v_cache + slot * p.cache_stride + h0 * L::ROW);
      continue;
    }
    Rot<D> rot;
    if (p.cos_sin != nullptr) load_rotation<D>(rot, p.cos_sin + pos * D, lane & 15u, p.interleaved);
    char *dst = (kind == 0 ? p.q_out + tok * p.q_out_stride : p.k_cache + slot * p.cache_stride) + h0 * L::ROW;
    finish_pairs<T, D, PR>(lo, hi, nh, kind == 0 ? p.q_weight : p.k_weight, p.eps, p.cos_sin != nullptr,
                           p.interleaved, rot, lane, dst);
  }
}

// ---------------------------------------------------------------------------
// TMA-staged kernel
// ---------------------------------------------------------------------------
constexpr uint32_t kQkvMaxStages = 16;
constexpr uint32_t kQkvMetaBytes = 32 * 16;  // per stage: int64 position and slot of up to 32 tokens
constexpr uint32_t kQkvBarrierBytes = 2 * kQkvMaxStages * 8;
constexpr uint64_t kQkvWaitNs = 2000000000ull;  // 2 s

// CW consumer warps, chunks of G heads.
template <typename T, int D, int G, int CW>
__global__ void __launch_bounds__(32 * (1 + CW), 1) qkv_tma_kernel(const __grid_constant__ QkvParams p) {
  constexpr uint32_t ROW_BYTES = D * 2;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t *full = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty = full + kQkvMaxStages;
  const uint32_t S = p.num_stages;
  unsigned char *stages = smem + kQkvBarrierBytes;
  const uint32_t warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t q_bytes = p.hq * ROW_BYTES;
  const uint32_t kv_bytes = p.hk * ROW_BYTES;
  const bool rope = p.cos_sin != nullptr;

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < S; ++s) {
      mbar_init(&full[s], 32);                  // every producer lane arrives
      mbar_init(&empty[s], CW);  // one arrival per consumer warp
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();  // Q/K/V may be written by the kernel just before this one

  if (warp == 0) {
    // producer: lane t handles token t of the tile.  The Q/K/V row copies go
    // out first (they need only the token index); the tile's slots and
    // positions were fetched one tile ahead, so only the cos/sin row copies
    // wait on a position.
    uint32_t iter = 0;
    int64_t next_slot = 0, next_pos = 0;
    auto fetch = [&](uint32_t tile) {
      const uint32_t tok = tile * p.tile_tokens + lane;
      if (tile < p.num_tiles && lane < p.tile_tokens && tok < p.num_tokens) {
        next_slot = p.slot64 ? load_int<int64_t>(p.slots, tok) : load_int<int32_t>(p.slots, tok);
        if (rope) next_pos = p.pos64 ? load_int<int64_t>(p.positions, tok) : load_int<int32_t>(p.positions, tok);
      }
    };
    fetch(blockIdx.x);
    for (uint32_t tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++iter) {
      const int64_t slot = next_slot, pos = next_pos;
      fetch(tile + gridDim.x);
      const uint32_t s = iter % S;
      if (iter >= S && !mbar_wait_bounded(&empty[s], ((iter / S) - 1) & 1u, kQkvWaitNs)) {
        if (lane == 0) raise_deverr(p.error_word, YL_DEVERR_TIMEOUT);
        break;
      }
      unsigned char *stage = stages + s * p.stage_bytes;
      int64_t *meta = reinterpret_cast<int64_t *>(stage);
      const uint32_t t0 = tile * p.tile_tokens;
      const uint32_t nt = min(p.tile_tokens, p.num_tokens - t0);
      unsigned char *dst = stage + kQkvMetaBytes + lane * p.token_bytes;
      const uint32_t tok = t0 + lane;
      if (lane == 0) mbar_expect_tx(&full[s], nt * (q_bytes + 2 * kv_bytes));
      __syncwarp();
      if (lane < nt) {
        if (q_bytes) bulk_load(dst, p.q + tok * p.q_stride, q_bytes, &full[s]);
        bulk_load(dst + q_bytes, p.k + tok * p.k_stride, kv_bytes, &full[s]);
        bulk_load(dst + q_bytes + kv_bytes, p.v + tok * p.v_stride, kv_bytes, &full[s]);
        meta[2 * lane] = pos;
        meta[2 * lane + 1] = slot;
      }
      const bool cos_row = rope && lane < nt && pos >= 0 && pos < p.max_position;
      const uint32_t cos_bytes = __popc(__ballot_sync(0xffffffffu, cos_row)) * D * 4u;
      if (lane == 0) mbar_arrive_expect_tx(&full[s], cos_bytes);
      __syncwarp();
      if (cos_row) bulk_load(dst + q_bytes + 2 * kv_bytes, p.cos_sin + pos * D, D * 4u, &full[s]);
      if (lane != 0) mbar_arrive(&full[s]);
    }
    // no copy may land after the CTA exits: wait for the phases armed last
    const uint32_t first = iter > S ? iter - S : 0;
    for (uint32_t j = first; j < iter; ++j) {
      if (!mbar_wait_bounded(&full[j % S], (j / S) & 1u, kQkvWaitNs)) {
        if (lane == 0) raise_deverr(p.error_word, YL_DEVERR_TIMEOUT);
        break;
      }
    }
    return;
  }

  // consumers
  using L = Lay<D>;
  constexpr int PR = G / 2;
  const uint32_t cw = warp - 1;
  const uint32_t lane_off = (lane & 15u) * L::SEG + (lane >> 4) * L::ROW;
  uint32_t iter = 0;
  for (uint32_t tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++iter) {
    const uint32_t s = iter % S;
    if (!mbar_wait_bounded(&full[s], (iter / S) & 1u, kQkvWaitNs)) {
      if (lane == 0) raise_deverr(p.error_word, YL_DEVERR_TIMEOUT);
      break;
    }
    const unsigned char *stage = stages + s * p.stage_bytes;
    const int64_t *meta = reinterpret_cast<const int64_t *>(stage);
    const uint32_t t0 = tile * p.tile_tokens;
    const uint32_t nt = min(p.tile_tokens, p.num_tokens - t0);
    for (uint32_t u = cw; u < nt * p.chunks; u += CW) {
      const uint32_t t = p.by_chunks.div(u);
      int kind;
      uint32_t h0, nh;
      chunk_heads(p, u - t * p.chunks, G, kind, h0, nh);
      const int64_t pos = meta[2 * t];
      const int64_t slot = meta[2 * t + 1];
      if (rope && (pos < 0 || pos >= p.max_position)) {
        if (lane == 0) raise_deverr(p.error_word, YL_DEVERR_POSITION_RANGE);
        continue;
      }
      if (kind != 0 && !slot_ok(p, slot, lane)) continue;
      const unsigned char *row = stage + kQkvMetaBytes + t * p.token_bytes;
      const char *src = reinterpret_cast<const char *>(row) + (kind == 0 ? 0u : (kind == 1 ? q_bytes : q_bytes + kv_bytes)) +
                        h0 * L::ROW + lane_off;
      Words<L::W> lo[PR], hi[PR];
#pragma unroll
      for (int pr = 0; pr < PR; ++pr)
        if (2 * pr + (lane >> 4) < nh) {
          load_words(lo[pr], src + 2 * pr * L::ROW);
          load_words(hi[pr], src + 2 * pr * L::ROW + L::HALF);
        }
      if (kind == 2) {
        copy_pairs<D, PR>(lo, hi, nh, lane, p.v_cache + slot * p.cache_stride + h0 * L::ROW);
        continue;
      }
      Rot<D> rot;
      if (rope)
        load_rotation<D>(rot, reinterpret_cast<const float *>(row + q_bytes + 2 * kv_bytes), lane & 15u,
                         p.interleaved);
      char *dst = (kind == 0 ? p.q_out + (t0 + t) * p.q_out_stride : p.k_cache + slot * p.cache_stride) + h0 * L::ROW;
      finish_pairs<T, D, PR>(lo, hi, nh, kind == 0 ? p.q_weight : p.k_weight, p.eps, rope, p.interleaved, rot, lane,
                             dst);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
}

int blocks_per_sm(const void *fn, size_t smem);  // kv_store.cu, at 256 threads

}  // namespace ylk

namespace {

using ylk::QkvParams;
using Kernel = void (*)(QkvParams);

// A TMA kernel shape: chunks of g heads, cw consumer warps.
struct TmaShape {
  Kernel fn;
  uint32_t g;
  uint32_t cw;
};

struct QkvKernels {
  Kernel small, big;
  uint32_t g_big;
  TmaShape tma[4];  // [0] is the default; YL_QKV_TMA_SHAPE picks another
};

template <typename T>
QkvKernels qkv_kernels(int head_dim) {
  using namespace ylk;
  switch (head_dim) {
    case 64:
      return {qkv_norm_rope_store_kernel<T, 64, 2>,
              qkv_norm_rope_store_kernel<T, 64, 8>,
              8,
              {{qkv_tma_kernel<T, 64, 8, 16>, 8, 16},
               {qkv_tma_kernel<T, 64, 4, 24>, 4, 24},
               {qkv_tma_kernel<T, 64, 4, 31>, 4, 31},
               {qkv_tma_kernel<T, 64, 2, 31>, 2, 31}}};
    case 128:
      return {qkv_norm_rope_store_kernel<T, 128, 2>,
              qkv_norm_rope_store_kernel<T, 128, 8>,
              8,
              {{qkv_tma_kernel<T, 128, 8, 16>, 8, 16},
               {qkv_tma_kernel<T, 128, 4, 24>, 4, 24},
               {qkv_tma_kernel<T, 128, 4, 31>, 4, 31},
               {qkv_tma_kernel<T, 128, 2, 31>, 2, 31}}};
    default:
      return {qkv_norm_rope_store_kernel<T, 256, 2>,
              qkv_norm_rope_store_kernel<T, 256, 4>,
              4,
              {{qkv_tma_kernel<T, 256, 4, 16>, 4, 16},
               {qkv_tma_kernel<T, 256, 2, 24>, 2, 24},
               {qkv_tma_kernel<T, 256, 2, 31>, 2, 31},
               {qkv_tma_kernel<T, 256, 2, 31>, 2, 31}}};
  }
}

// YL_QKV_STAGES=2..16 sets the TMA kernel's number of stages (default 6:
// 3 to 8 measured within 3 % of each other at prefill sizes, 12 and more
// slower).
uint32_t qkv_stages() {
  static const uint32_t v = [] {
    const char *e = std::getenv("YL_QKV_STAGES");
    const int i = e ? std::atoi(e) : 6;
    return static_cast<uint32_t>(i >= 2 && i <= static_cast<int>(ylk::kQkvMaxStages) ? i : 6);
  }();
  return v;
}

// YL_QKV_TMA_SHAPE=0..3 picks a TMA kernel shape (for tuning runs).
int qkv_tma_shape() {
  static const int v = [] {
    const char *e = std::getenv("YL_QKV_TMA_SHAPE");
    const int i = e ? std::atoi(e) : 0;
    return i >= 0 && i < 4 ? i : 0;
  }();
  return v;
}

void set_chunks(QkvParams &p, uint32_t G) {
  p.cq = (p.hq + G - 1) / G;
  p.ck = (p.hk + G - 1) / G;
  p.chunks = p.cq + 2 * p.ck;
  p.by_chunks = ylk::FastDiv(p.chunks);
}

// YL_QKV_ENGINE=register|tma overrides the per-launch choice (for tests).
int qkv_engine_override() {
  static const int v = [] {
    const char *e = std::getenv("YL_QKV_ENGINE");
    if (e == nullptr) return 0;
    if (std::string(e) == "register") return 1;
    if (std::string(e) == "tma") return 2;
    return 0;
  }();
  return v;
}

}  // namespace

extern "C" int yl_qkv_norm_rope_store(const yl_qkv_store_args *a, cudaStream_t stream) {
  using namespace ylk;
  clear_last_error();
  if (a == nullptr) return fail(YL_ERR_NULL_ARG, "yl_qkv_norm_rope_store: args is NULL");
  if (a->num_tokens < 0) return fail(YL_ERR_BAD_SIZE, "yl_qkv_norm_rope_store: num_tokens=%lld < 0", a->num_tokens);
  if (a->dtype != YL_DTYPE_BF16 && a->dtype != YL_DTYPE_F16)
    return fail(YL_ERR_BAD_SIZE, "yl_qkv_norm_rope_store: dtype=%lld is not bf16 (0) or fp16 (1)", a->dtype);
  if (a->head_dim != 64 && a->head_dim != 128 && a->head_dim != 256)
    return fail(YL_ERR_UNSUPPORTED, "yl_qkv_norm_rope_store: head_dim=%lld is not 64, 128 or 256", a->head_dim);
  if (a->num_q_heads < 0 || a->num_kv_heads <= 0)
    return fail(YL_ERR_BAD_SIZE, "yl_qkv_norm_rope_store: num_q_heads=%lld, num_kv_heads=%lld", a->num_q_heads,
                a->num_kv_heads);
  if ((a->slot_is_int64 | a->position_is_int64 | a->rope_interleaved) & ~1)
    return fail(YL_ERR_BAD_SIZE, "yl_qkv_norm_rope_store: slot_is_int64, position_is_int64 and rope_interleaved "
                                 "must be 0 or 1");
  if (!(a->eps >= 0.f) || !std::isfinite(a->eps))
    return fail(YL_ERR_BAD_SIZE, "yl_qkv_norm_rope_store: eps must be finite and >= 0");
  if (a->num_tokens == 0) return YL_OK;
  if (!a->k || !a->v || !a->k_cache || !a->v_cache || !a->slots)
    return fail(YL_ERR_NULL_ARG, "yl_qkv_norm_rope_store: k, v, k_cache, v_cache and slots must be non-NULL");
  if (a->num_q_heads > 0 && (!a->q || !a->q_out))
    return fail(YL_ERR_NULL_ARG, "yl_qkv_norm_rope_store: q and q_out must be non-NULL when num_q_heads > 0");
  if (a->cos_sin_cache && (!a->positions || a->max_position <= 0))
    return fail(YL_ERR_BAD_SIZE, "yl_qkv_norm_rope_store: cos_sin_cache needs positions and max_position=%lld > 0",
                a->max_position);
  const int64_t D = a->head_dim;
  const int64_t q_row = a->num_q_heads * D * 2, kv_row = a->num_kv_heads * D * 2;
  if ((a->num_q_heads > 0 && (a->q_row_stride < q_row || a->q_out_row_stride < q_row)) ||
      a->k_row_stride < kv_row || a->v_row_stride < kv_row || a->cache_row_stride < kv_row)
    return fail(YL_ERR_BAD_SIZE, "yl_qkv_norm_rope_store: a row stride is below its row (%lld B per K/V row)", kv_row);
  const uint64_t heads = static_cast<uint64_t>(a->num_q_heads) + 2ull * static_cast<uint64_t>(a->num_kv_heads);
  if (static_cast<uint64_t>(a->num_tokens) * heads >= (1ull << 31) || a->num_tokens >= (1ll << 31))
    return fail(YL_ERR_UNSUPPORTED, "yl_qkv_norm_rope_store: num_tokens=%lld x heads exceeds 2^31 rows",
                a->num_tokens);
  // every row base, stride and weight is a multiple of one lane's vector
  const uintptr_t vec = static_cast<uintptr_t>(D / 16);
  uintptr_t bits = reinterpret_cast<uintptr_t>(a->k) | reinterpret_cast<uintptr_t>(a->v) |
                   reinterpret_cast<uintptr_t>(a->k_cache) | reinterpret_cast<uintptr_t>(a->v_cache) |
                   static_cast<uintptr_t>(a->k_row_stride) | static_cast<uintptr_t>(a->v_row_stride) |
                   static_cast<uintptr_t>(a->cache_row_stride) | reinterpret_cast<uintptr_t>(a->q_weight) |
                   reinterpret_cast<uintptr_t>(a->k_weight);
  if (a->num_q_heads > 0)
    bits |= reinterpret_cast<uintptr_t>(a->q) | reinterpret_cast<uintptr_t>(a->q_out) |
            static_cast<uintptr_t>(a->q_row_stride) | static_cast<uintptr_t>(a->q_out_row_stride);
  if ((bits & (vec - 1)) != 0 || (reinterpret_cast<uintptr_t>(a->cos_sin_cache) & 15u) != 0 ||
      (reinterpret_cast<uintptr_t>(a->slots) & (a->slot_is_int64 ? 7u : 3u)) != 0 ||
      (a->cos_sin_cache && (reinterpret_cast<uintptr_t>(a->positions) & (a->position_is_int64 ? 7u : 3u)) != 0))
    return fail(YL_ERR_ALIGNMENT,
                "yl_qkv_norm_rope_store: rows, strides and weights must be %lld-byte aligned, cos_sin_cache 16-byte, "
                "slots/positions to their element size",
                static_cast<long long>(vec));

  QkvParams p{};
  p.q = static_cast<const char *>(a->q);
  p.k = static_cast<const char *>(a->k);
  p.v = static_cast<const char *>(a->v);
  p.q_out = static_cast<char *>(a->q_out);
  p.k_cache = static_cast<char *>(a->k_cache);
  p.v_cache = static_cast<char *>(a->v_cache);
  p.slots = a->slots;
  p.q_weight = static_cast<const char *>(a->q_weight);
  p.k_weight = static_cast<const char *>(a->k_weight);
  p.cos_sin = a->cos_sin_cache;
  p.positions = a->positions;
  p.q_stride = a->q_row_stride;
  p.k_stride = a->k_row_stride;
  p.v_stride = a->v_row_stride;
  p.q_out_stride = a->q_out_row_stride;
  p.cache_stride = a->cache_row_stride;
  p.num_slots = a->num_slots;
  p.max_position = a->max_position;
  p.error_word = a->error_word;
  p.num_tokens = static_cast<uint32_t>(a->num_tokens);
  p.hq = static_cast<uint32_t>(a->num_q_heads);
  p.hk = static_cast<uint32_t>(a->num_kv_heads);
  p.eps = a->eps;
  p.slot64 = a->slot_is_int64;
  p.pos64 = a->position_is_int64;
  p.interleaved = a->rope_interleaved;

  const QkvKernels ks = a->dtype == YL_DTYPE_BF16 ? qkv_kernels<__nv_bfloat16>(a->head_dim) : qkv_kernels<__half>(a->head_dim);
  const uint64_t sms = static_cast<uint64_t>(sm_count());

  // The TMA kernel when the batch is large (its tiles cover every SM several
  // times and the chunks fill the register kernel's warp slots twice over)
  // and its bulk copies are legal: 16-byte aligned sources and strides, and
  // one token's rows fit a stage.
  const uint64_t token_bytes = static_cast<uint64_t>(q_row + 2 * kv_row) + (a->cos_sin_cache ? D * 4 : 0);
  // S stages of equal size share 227 KB of shared memory; a stage holds
  // tile_tokens whole tokens (at most 32, at least 1, else no TMA kernel)
  uint32_t S = qkv_stages();
  uint64_t tile_tokens = 0;
  for (; S >= 2; --S) {
    const uint64_t stage_budget = (227u * 1024u - kQkvBarrierBytes) / S;
    tile_tokens = stage_budget > kQkvMetaBytes + 127 ? (stage_budget - kQkvMetaBytes - 127) / token_bytes : 0;
    if (tile_tokens >= 1) break;
  }
  if (tile_tokens > 32) tile_tokens = 32;
  const uintptr_t bulk_bits = reinterpret_cast<uintptr_t>(a->k) | reinterpret_cast<uintptr_t>(a->v) |
                              static_cast<uintptr_t>(a->k_row_stride) | static_cast<uintptr_t>(a->v_row_stride) |
                              (a->num_q_heads > 0 ? reinterpret_cast<uintptr_t>(a->q) |
                                                        static_cast<uintptr_t>(a->q_row_stride)
                                                  : 0);
  const bool tma_legal = tile_tokens >= 1 && (bulk_bits & 15u) == 0;
  const uint64_t chunks_big = (p.hq + ks.g_big - 1) / ks.g_big + 2 * ((p.hk + ks.g_big - 1) / ks.g_big);
  const uint64_t slots_big = sms * blocks_per_sm(reinterpret_cast<const void *>(ks.big), 0) * 8;
  const bool large = static_cast<uint64_t>(a->num_tokens) * chunks_big >= 2 * slots_big;
  const uint64_t tiles = tma_legal ? (static_cast<uint64_t>(a->num_tokens) + tile_tokens - 1) / tile_tokens : 0;
  int engine = large ? (tma_legal && tiles >= 2 * sms ? 2 : 1) : 0;
  if (qkv_engine_override() == 1) engine = large ? 1 : 0;
  if (qkv_engine_override() == 2 && tma_legal) engine = 2;

  if (engine == 2) {
    const TmaShape &shape = ks.tma[qkv_tma_shape()];
    set_chunks(p, shape.g);
    p.tile_tokens = static_cast<uint32_t>(tile_tokens);
    p.num_tiles = static_cast<uint32_t>(tiles);
    p.token_bytes = static_cast<uint32_t>(token_bytes);
    p.stage_bytes = static_cast<uint32_t>((kQkvMetaBytes + tile_tokens * token_bytes + 127) / 128 * 128);
    p.num_stages = S;
    const size_t smem = kQkvBarrierBytes + static_cast<size_t>(S) * p.stage_bytes;
    if (cudaFuncSetAttribute(shape.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess)
      return check_launch("yl_qkv_norm_rope_store: shared memory attribute");
    const uint64_t grid = tiles < sms ? tiles : sms;
    return launch_dependent(shape.fn, dim3(static_cast<unsigned>(grid)), dim3(32 * (1 + shape.cw)), smem, stream,
                            "yl_qkv_norm_rope_store launch", p);
  }
  const Kernel fn = engine == 1 ? ks.big : ks.small;
  set_chunks(p, engine == 1 ? ks.g_big : 2);
  p.items = static_cast<uint32_t>(a->num_tokens * static_cast<int64_t>(p.chunks));
  const uint64_t want = (static_cast<uint64_t>(p.items) + 7) / 8;  // 8 warps per block
  const uint64_t cap = sms * blocks_per_sm(reinterpret_cast<const void *>(fn), 0);
  return launch_dependent(fn, dim3(static_cast<unsigned>(want < cap ? want : cap)), dim3(256), 0, stream,
                          "yl_qkv_norm_rope_store launch", p);
}
