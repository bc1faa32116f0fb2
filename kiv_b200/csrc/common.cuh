// Shared device helpers for the KIV sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/kiv_b200.h"

#define KIV_FULL_MASK 0xffffffffu

namespace kiv {

// ---------------------------------------------------------------------------
// element types: 16-byte vectors of V elements
// ---------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static constexpr int V = 4;
  __device__ __forceinline__ static void unpack(const uint4 &u, float *f) {
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
  }
  __device__ __forceinline__ static uint4 pack(const float *f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]),
                      __float_as_uint(f[2]), __float_as_uint(f[3]));
  }
  __device__ __forceinline__ static float to_f(float x) { return x; }
  __device__ __forceinline__ static float from_f(float x) { return x; }
};
template <> struct Elem<__nv_bfloat16> {
  static constexpr int V = 8;
  __device__ __forceinline__ static void unpack(const uint4 &u, float *f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  __device__ __forceinline__ static uint4 pack(const float *f) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t *>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
  __device__ __forceinline__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};
template <> struct Elem<__half> {
  static constexpr int V = 8;
  __device__ __forceinline__ static void unpack(const uint4 &u, float *f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2 *>(&w[i]);
      float2 p = __half22float2(h);
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    }
  }
  __device__ __forceinline__ static uint4 pack(const float *f) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t *>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
  __device__ __forceinline__ static float to_f(__half x) { return __half2float(x); }
  __device__ __forceinline__ static __half from_f(float x) { return __float2half_rn(x); }
};

__device__ __forceinline__ uint4 ld16(const void *p) { return *reinterpret_cast<const uint4 *>(p); }
__device__ __forceinline__ uint4 ld16_stream(const void *p) {
  // streaming read: the K/V rows of the cold tier are touched once per step
  return __ldcs(reinterpret_cast<const uint4 *>(p));
}
__device__ __forceinline__ void st16(void *p, const uint4 &v) { *reinterpret_cast<uint4 *>(p) = v; }

// ---------------------------------------------------------------------------
// order-preserving float <-> uint32 keys (larger float -> larger key)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t f2key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

// ---------------------------------------------------------------------------
// group transpose-reduce.  A group of LPR consecutive lanes each holds N
// partial sums (one per query row).  After the call, lane l of the group
// holds the full sum of NOUT = max(1, N / LPR) rows starting at `base`,
// in v[0 .. NOUT).  N and LPR are powers of two.
// ---------------------------------------------------------------------------
template <int N, int O>
__device__ __forceinline__ void tr_reduce(float *v, int lane, int &base) {
  if constexpr (O == 0) {
    return;
  } else if constexpr (N == 1) {
    v[0] += __shfl_xor_sync(KIV_FULL_MASK, v[0], O);
    tr_reduce<1, O / 2>(v, lane, base);
  } else {
    constexpr int H = N / 2;
    const bool hi = (lane & O) != 0;
#pragma unroll
    for (int i = 0; i < H; ++i) {
      float send = hi ? v[i] : v[i + H];
      float keep = hi ? v[i + H] : v[i];
      v[i] = keep + __shfl_xor_sync(KIV_FULL_MASK, send, O);
    }
    if (hi) base += H;
    tr_reduce<H, O / 2>(v, lane, base);
  }
}

template <int O>
__device__ __forceinline__ float group_max(float x) {
  if constexpr (O == 0) {
    return x;
  } else {
    x = fmaxf(x, __shfl_xor_sync(KIV_FULL_MASK, x, O));
    return group_max<O / 2>(x);
  }
}

// ---------------------------------------------------------------------------
// Dot products of one head_dim row against RCH query rows.  The row is split
// over a group of LPR lanes; each lane owns VPL 16-byte vectors (vector index
// g + j*LPR, j < VPL, for lane g of the group), so a group load of one row is
// fully coalesced.  `nv` = head_dim / V (vectors in a row).
// ---------------------------------------------------------------------------
template <typename T, int LPR, int VPL, int RCH>
struct RowDot {
  static constexpr int V = Elem<T>::V;
  float q[RCH][VPL * V];

  // rows[r] == nullptr -> zero row (padding)
  __device__ __forceinline__ void load_query(const T *const *rows, int g, int nv, float scale) {
#pragma unroll
    for (int r = 0; r < RCH; ++r) {
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const int vi = g + j * LPR;
        float f[V];
        if (rows[r] != nullptr && vi < nv) {
          Elem<T>::unpack(ld16(rows[r] + vi * V), f);
        } else {
#pragma unroll
          for (int e = 0; e < V; ++e) f[e] = 0.f;
        }
#pragma unroll
        for (int e = 0; e < V; ++e) q[r][j * V + e] = f[e] * scale;
      }
    }
  }

  // rows[r]: fp32 rows in shared memory (nullptr -> zero row)
  __device__ __forceinline__ void load_query_f32(const float *const *rows, int g, int nv) {
#pragma unroll
    for (int r = 0; r < RCH; ++r) {
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const int vi = g + j * LPR;
#pragma unroll
        for (int e = 0; e < V; e += 4) {
          float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
          if (rows[r] != nullptr && vi < nv) f = *reinterpret_cast<const float4 *>(rows[r] + vi * V + e);
          q[r][j * V + e] = f.x;
          q[r][j * V + e + 1] = f.y;
          q[r][j * V + e + 2] = f.z;
          q[r][j * V + e + 3] = f.w;
        }
      }
    }
  }

  // partial dots of this lane's slice of `row` (nullptr -> zeros)
  template <bool STREAM>
  __device__ __forceinline__ void partial(const T *row, int g, int nv, float (&acc)[RCH]) const {
    float2 a2[RCH];
#pragma unroll
    for (int r = 0; r < RCH; ++r) a2[r] = make_float2(0.f, 0.f);
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int vi = g + j * LPR;
      if (row != nullptr && vi < nv) {
        float f[V];
        Elem<T>::unpack(STREAM ? ld16_stream(row + vi * V) : ld16(row + vi * V), f);
#pragma unroll
        for (int e = 0; e < V; e += 2) {
          const float2 k2 = make_float2(f[e], f[e + 1]);
#pragma unroll
          for (int r = 0; r < RCH; ++r) {
            const float2 q2 = make_float2(q[r][j * V + e], q[r][j * V + e + 1]);
            a2[r] = __ffma2_rn(q2, k2, a2[r]);
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < RCH; ++r) acc[r] = a2[r].x + a2[r].y;
  }
};

// number of output rows a lane holds after tr_reduce<RCH, LPR/2>
template <int RCH, int LPR>
struct TrOut {
  static constexpr int N = (RCH / LPR) > 0 ? (RCH / LPR) : 1;
  static constexpr int REPL = (LPR / RCH) > 0 ? (LPR / RCH) : 1;  // lanes sharing a row
};

// ---------------------------------------------------------------------------
// device state access
// ---------------------------------------------------------------------------
__device__ __forceinline__ int64_t st_ld(const int64_t *st, int w) {
  return *reinterpret_cast<const volatile int64_t *>(st + w);
}

// last-block-done pattern: returns true in exactly one block, after every
// block of the grid has passed this point.  Counter is reset by the winner.
__device__ __forceinline__ bool last_block(unsigned long long *ctr, unsigned long long nblocks) {
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned long long prev = atomicAdd(ctr, 1ull);
    s_last = (prev == nblocks - 1) ? 1 : 0;
  }
  __syncthreads();
  if (s_last) {
    __threadfence();
    if (threadIdx.x == 0) *ctr = 0ull;
  }
  return s_last != 0;
}

// programmatic dependent launch: wait for the preceding kernel's results,
// then let the next kernel in the stream start its prologue.
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

}  // namespace kiv

namespace kiv {

// ---------------------------------------------------------------------------
// 1-D bulk copies (cp.async.bulk, TMA engine, no tensor map, one destination CTA)
// completing on an mbarrier.  Waits are bounded: after ~2^31 cycles the wait
// gives up and reports failure so the kernel can set an error bit and leave.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > (1ll << 31)) return false;
  }
  return true;
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

}  // namespace kiv
