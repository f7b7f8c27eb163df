// One layer's attention input in one pass, for sm_100a: per-head RMSNorm of Q
// and K, rotary embedding of Q and K, Q written out, K and V stored into the
// paged pool by slot.
//
// Work item = one (token, head) row of head_dim elements, enumerated
// token-major over the token's Q heads, then K heads, then V heads, so
// consecutive warps read consecutive bytes of one token's QKV row.  One warp
// per item: lane l holds elements [l * EPL, (l + 1) * EPL), EPL = head_dim /
// 32, as one 4/8/16-byte vector.  The sum of squares is a warp all-reduce;
// for neox rotation element j pairs with j + head_dim / 2, which sits in lane
// l ^ 16 at the same register, so the partner comes from one shuffle; GPT-J
// pairs (2j, 2j + 1) sit in the same lane.
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

#include "common.cuh"

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
  uint32_t items;  // N * (Hq + 2 Hk)  (< 2^31)
  uint32_t hq;
  uint32_t hk;
  uint32_t heads;  // Hq + 2 Hk
  FastDiv by_heads;
  float eps;
  int slot64;
  int pos64;
  int interleaved;
};

template <typename T>
struct Elem;
template <>
struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_float(uint32_t bits) {
    return __bfloat162float(__ushort_as_bfloat16(static_cast<unsigned short>(bits)));
  }
  static __device__ __forceinline__ uint32_t from_float(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
  }
};
template <>
struct Elem<__half> {
  static __device__ __forceinline__ float to_float(uint32_t bits) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits)));
  }
  static __device__ __forceinline__ uint32_t from_float(float f) { return __half_as_ushort(__float2half_rn(f)); }
};

// A lane's EPL 16-bit elements as EPL / 2 32-bit words.
template <int WORDS>
struct Words {
  uint32_t w[WORDS];
};

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

// Weights are read by every row: cached path.
template <int WORDS>
__device__ __forceinline__ void load_cached(Words<WORDS> &x, const char *p) {
  if constexpr (WORDS == 1) {
    x.w[0] = __ldg(reinterpret_cast<const uint32_t *>(p));
  } else if constexpr (WORDS == 2) {
    const uint2 t = __ldg(reinterpret_cast<const uint2 *>(p));
    x.w[0] = t.x, x.w[1] = t.y;
  } else {
    const uint4 t = __ldg(reinterpret_cast<const uint4 *>(p));
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
    out[0] = __ldg(p);
  } else if constexpr (N == 2) {
    const float2 t = __ldg(reinterpret_cast<const float2 *>(p));
    out[0] = t.x, out[1] = t.y;
  } else {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
      const float4 t = __ldg(reinterpret_cast<const float4 *>(p + i));
      out[i] = t.x, out[i + 1] = t.y, out[i + 2] = t.z, out[i + 3] = t.w;
    }
  }
}

template <typename IntT>
__device__ __forceinline__ int64_t load_int(const void *p, uint32_t i) {
  return static_cast<int64_t>(__ldg(static_cast<const IntT *>(p) + i));
}

template <typename T, int D>
__global__ void __launch_bounds__(256) qkv_norm_rope_store_kernel(const __grid_constant__ QkvParams p) {
  constexpr int EPL = D / 32;
  constexpr int WORDS = EPL / 2;
  constexpr int ROW_BYTES = D * 2;
  using E = Elem<T>;
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint32_t num_warps = (gridDim.x * blockDim.x) >> 5;
  const uint32_t lane_off = lane * EPL * 2;
  pdl_wait();  // Q/K/V may be written by the kernel just before this one
  for (uint32_t item = warp; item < p.items; item += num_warps) {
    const uint32_t tok = p.by_heads.div(item);
    const uint32_t h = item - tok * p.heads;
    const int kind = h < p.hq ? 0 : (h < p.hq + p.hk ? 1 : 2);  // Q, K, V
    const uint32_t hh = kind == 0 ? h : (kind == 1 ? h - p.hq : h - p.hq - p.hk);
    const char *src = kind == 0 ? p.q + tok * p.q_stride : (kind == 1 ? p.k + tok * p.k_stride : p.v + tok * p.v_stride);
    Words<WORDS> x;
    load_once(x, src + hh * ROW_BYTES + lane_off);
    int64_t slot = 0;
    if (kind != 0) slot = p.slot64 ? load_int<int64_t>(p.slots, tok) : load_int<int32_t>(p.slots, tok);
    int64_t pos = 0;
    if (p.cos_sin != nullptr) {
      pos = p.pos64 ? load_int<int64_t>(p.positions, tok) : load_int<int32_t>(p.positions, tok);
      if (pos < 0 || pos >= p.max_position) {
        if (lane == 0) raise_deverr(p.error_word, YL_DEVERR_POSITION_RANGE);
        continue;
      }
    }
    bool store_ok = true;
    if (kind != 0) {
      store_ok = slot >= 0 && (p.num_slots <= 0 || slot < p.num_slots);
      if (!store_ok && slot != -1 && lane == 0) raise_deverr(p.error_word, YL_DEVERR_SLOT_RANGE);
    }
    if (kind == 2) {
      if (store_ok) store_words(p.v_cache + slot * p.cache_stride + hh * ROW_BYTES + lane_off, x);
      continue;
    }

    float f[EPL];
#pragma unroll
    for (int i = 0; i < WORDS; ++i) {
      f[2 * i] = E::to_float(x.w[i] & 0xffffu);
      f[2 * i + 1] = E::to_float(x.w[i] >> 16);
    }
    const char *w = kind == 0 ? p.q_weight : p.k_weight;
    if (w != nullptr) {
      Words<WORDS> wv;
      load_cached(wv, w + lane_off);
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < EPL; ++i) ss += f[i] * f[i];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float r = rsqrtf(ss / static_cast<float>(D) + p.eps);
#pragma unroll
      for (int i = 0; i < WORDS; ++i) {
        // the norm's output is a T tensor in the unfused sequence: round here
        f[2 * i] = E::to_float(E::from_float(f[2 * i] * r * E::to_float(wv.w[i] & 0xffffu)));
        f[2 * i + 1] = E::to_float(E::from_float(f[2 * i + 1] * r * E::to_float(wv.w[i] >> 16)));
      }
    }
    if (p.cos_sin != nullptr) {
      const float *cs = p.cos_sin + pos * D;
      if (!p.interleaved) {
        // neox: y_j = x_j c_j - x_{j+D/2} s_j,  y_{j+D/2} = x_{j+D/2} c_j + x_j s_j
        float c[EPL], s[EPL];
        const uint32_t j0 = (lane & 15u) * EPL;
        load_floats(c, cs + j0);
        load_floats(s, cs + D / 2 + j0);
        const float sign = lane < 16 ? -1.f : 1.f;
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
          const float partner = __shfl_xor_sync(0xffffffffu, f[i], 16);
          f[i] = f[i] * c[i] + sign * partner * s[i];
        }
      } else {
        // GPT-J: y_{2j} = x_{2j} c_j - x_{2j+1} s_j,  y_{2j+1} = x_{2j+1} c_j + x_{2j} s_j
        float c[EPL / 2], s[EPL / 2];
        const uint32_t j0 = lane * (EPL / 2);
        load_floats(c, cs + j0);
        load_floats(s, cs + D / 2 + j0);
#pragma unroll
        for (int i = 0; i < EPL / 2; ++i) {
          const float a = f[2 * i], b = f[2 * i + 1];
          f[2 * i] = a * c[i] - b * s[i];
          f[2 * i + 1] = b * c[i] + a * s[i];
        }
      }
    }
    Words<WORDS> y;
#pragma unroll
    for (int i = 0; i < WORDS; ++i) y.w[i] = E::from_float(f[2 * i]) | (E::from_float(f[2 * i + 1]) << 16);
    if (kind == 0) {
      store_words(p.q_out + tok * p.q_out_stride + hh * ROW_BYTES + lane_off, y);
    } else if (store_ok) {
      store_words(p.k_cache + slot * p.cache_stride + hh * ROW_BYTES + lane_off, y);
    }
  }
}

int blocks_per_sm(const void *fn, size_t smem);  // kv_store.cu, at 256 threads

}  // namespace ylk

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
  if (static_cast<uint64_t>(a->num_tokens) * heads >= (1ull << 31))
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

  QkvParams p;
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
  p.hq = static_cast<uint32_t>(a->num_q_heads);
  p.hk = static_cast<uint32_t>(a->num_kv_heads);
  p.heads = static_cast<uint32_t>(heads);
  p.items = static_cast<uint32_t>(a->num_tokens * static_cast<int64_t>(heads));
  p.by_heads = FastDiv(p.heads);
  p.eps = a->eps;
  p.slot64 = a->slot_is_int64;
  p.pos64 = a->position_is_int64;
  p.interleaved = a->rope_interleaved;

  using Kernel = void (*)(QkvParams);
  const bool bf16 = a->dtype == YL_DTYPE_BF16;
  Kernel fn;
  switch (a->head_dim) {
    case 64: fn = bf16 ? qkv_norm_rope_store_kernel<__nv_bfloat16, 64> : qkv_norm_rope_store_kernel<__half, 64>; break;
    case 128: fn = bf16 ? qkv_norm_rope_store_kernel<__nv_bfloat16, 128> : qkv_norm_rope_store_kernel<__half, 128>; break;
    default: fn = bf16 ? qkv_norm_rope_store_kernel<__nv_bfloat16, 256> : qkv_norm_rope_store_kernel<__half, 256>; break;
  }
  const uint64_t want = (static_cast<uint64_t>(p.items) + 7) / 8;  // 8 warps per block
  const uint64_t cap = static_cast<uint64_t>(sm_count()) * blocks_per_sm(reinterpret_cast<const void *>(fn), 0);
  fn<<<static_cast<unsigned>(want < cap ? want : cap), 256, 0, stream>>>(p);
  return check_launch("yl_qkv_norm_rope_store launch");
}
