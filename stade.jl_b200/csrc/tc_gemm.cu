// Tensor-core (tcgen05 / TMEM) Float32 contractions of the mlp2_ce adjoint,
// with 3xTF32 splitting so that the products keep Float32 accuracy.
//
// C[m, n] = sum_k A[m, k] B[n, k] on 5th-generation tensor cores:
//   - 8 "transform" warps load 128 x 32 Float32 tiles of A and B from global
//     memory (16-byte coalesced loads), split every value into
//     hi = a with the low 13 mantissa bits cleared (exactly representable in
//     TF32) and lo = a - hi (exact), and store hi and lo tiles into shared
//     memory in the canonical K-major 128-byte-swizzled UMMA layout;
//   - one thread of a 9th warp issues tcgen05.mma.kind::tf32 (M = 128,
//     N = 128, K = 8) three times per K step: hi*hi, hi*lo, lo*hi (the lo*lo
//     term is below Float32 rounding); the accumulator lives in TMEM;
//   - shared-memory stages are handed back by tcgen05.commit on an mbarrier;
//   - after the last K block the 8 warps read the accumulator with
//     tcgen05.ld and apply the fused epilogue.
// Every mbarrier wait is bounded (about two seconds of clock): on timeout
// the kernel records an error in g_tc_error, skips the remaining work, waits
// (bounded) for its own tensor-core operations and frees its TMEM.
//
// tcgen05 has no f64 kind and mixing operand types in one kind::f16 MMA is
// invalid, so this file handles Float32 only.
#include <cstdint>
#include <cstdlib>
#include <cstring>

#include "tc_gemm.cuh"

namespace stade {
namespace tc {

constexpr int BM = 128, BN = 128, BK = 32, STAGES = 3;
constexpr int kXWarps = 8;                   // transform + epilogue warps
constexpr int kMmaWarp = kXWarps;            // warp 8 issues MMAs, owns TMEM
constexpr int kThreads = (kXWarps + 1) * 32; // 288
constexpr int kTileBytes = 128 * BK * 4;     // 16 KiB (128 rows x 128 bytes)
constexpr int kStageBytes = 4 * kTileBytes;  // A hi, A lo, B hi, B lo
constexpr int kSmemBytes = STAGES * kStageBytes + 1024 + 256;
constexpr uint32_t kTmemCols = 128;
constexpr long long kWaitCycles = 4000000000LL;  // ~2 s at 1.9 GHz

__device__ int g_tc_error = 0;

// ---- PTX wrappers -------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false (and the error flag set) when the phase does not
// complete within kWaitCycles.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try(bar, parity)) {
    if (clock64() - t0 > kWaitCycles) {
      atomicExch(&g_tc_error, 1);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t slot_addr) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_addr),
               "r"(kTmemCols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(kTmemCols)
               : "memory");
}
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}
// 32 lanes x 32 columns of 32-bit accumulator: thread i of the warp gets row
// (lane base + i), columns col .. col + 31.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (tcgen05 matrix-descriptor format, version 1).
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);  // start address / 16
  d |= (uint64_t)1u << 16;                  // leading-dimension offset (unused here)
  d |= (uint64_t)(1024u >> 4) << 32;        // stride-dimension offset / 16
  d |= (uint64_t)1u << 46;                  // descriptor version
  d |= (uint64_t)2u << 61;                  // 128-byte swizzle
  return d;
}
// Instruction descriptor of kind::tf32: D f32, A/B tf32, both K-major, M x N.
constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

// Byte offset of the 16-byte chunk c (k = 4c .. 4c+3) of row r in a
// 128-row x 128-byte tile with the 128-byte swizzle.
__device__ __forceinline__ uint32_t tile_off(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ float tf32_hi(float a) {
  return __uint_as_float(__float_as_uint(a) & 0xFFFFE000u);
}

__device__ __forceinline__ void st_split(uint8_t* hi, uint8_t* lo, uint32_t off, float4 v) {
  float4 h, l;
  h.x = tf32_hi(v.x); l.x = v.x - h.x;
  h.y = tf32_hi(v.y); l.y = v.y - h.y;
  h.z = tf32_hi(v.z); l.z = v.z - h.z;
  h.w = tf32_hi(v.w); l.w = v.w - h.w;
  *reinterpret_cast<float4*>(hi + off) = h;
  *reinterpret_cast<float4*>(lo + off) = l;
}

// ---- operand loaders (one tile of up to 128 rows x 32 k, 256 threads) -----------
// `tile_rows` (<= 128) is the tile height: 128 for A, BN for B.
// K-contiguous source: element (r, k) = p[r * ld + k]. Thread t takes 4
// float4, idx = t + 256 i: row idx / 8, chunk idx % 8 (eight threads read one
// 128-byte row segment; their swizzled stores hit eight different banks).
struct LoadK {
  const float* p;
  int ld, rows, K;
  int ones_row;  // unused for K-contiguous sources
  __device__ __forceinline__ void load(int r0, int k0, int t, int tile_rows, float4 (&v)[4]) const {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = t + 256 * i;
      const int rr = idx >> 3;
      const int r = r0 + rr, k = k0 + 4 * (idx & 7);
      if (rr >= tile_rows) {
        v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      } else if (r < rows && k + 3 < K) {
        v[i] = __ldg(reinterpret_cast<const float4*>(p + (int64_t)r * ld + k));
      } else {
        float e[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) e[q] = (r < rows && k + q < K) ? p[(int64_t)r * ld + k + q] : 0.f;
        v[i] = make_float4(e[0], e[1], e[2], e[3]);
      }
    }
  }
  __device__ __forceinline__ void store(uint8_t* hi, uint8_t* lo, int t, int tile_rows,
                                        const float4 (&v)[4]) const {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = t + 256 * i;
      if ((idx >> 3) < tile_rows) st_split(hi, lo, tile_off(idx >> 3, idx & 7), v[i]);
    }
  }
};

// Row-contiguous source: element (r, k) = p[k * ld + r] (the tile is the
// transpose of a stored block). Thread t (warp w, lane l) takes rows
// 4l .. 4l+3 of chunk w: four float4 loads along r (a warp reads 512
// contiguous bytes per k), a 4 x 4 register transpose, four swizzled chunk
// stores (row order rotated by l / 2 so a quarter-warp hits eight banks).
// `ones_row` (>= 0) reads as 1.0 on that row and 0 past `rows`.
struct LoadMN {
  const float* p;
  int ld, rows, K;
  int ones_row;
  __device__ __forceinline__ float elem(int r, int k) const {
    if (k >= K) return 0.f;
    if (r == ones_row) return 1.f;
    return r < rows ? p[(int64_t)k * ld + r] : 0.f;
  }
  __device__ __forceinline__ void load(int r0, int k0, int t, int tile_rows, float4 (&v)[4]) const {
    const int w = t >> 5, l = t & 31;
    const int r = r0 + 4 * l;
    const bool in_tile = 4 * l < tile_rows;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int k = k0 + 4 * w + q;
      if (!in_tile) {
        v[q] = make_float4(0.f, 0.f, 0.f, 0.f);
      } else if (k < K && r + 3 < rows && (ones_row < r || ones_row > r + 3)) {
        v[q] = __ldg(reinterpret_cast<const float4*>(p + (int64_t)k * ld + r));
      } else {
        v[q] = make_float4(elem(r, k), elem(r + 1, k), elem(r + 2, k), elem(r + 3, k));
      }
    }
  }
  __device__ __forceinline__ void store(uint8_t* hi, uint8_t* lo, int t, int tile_rows,
                                        const float4 (&v)[4]) const {
    const int w = t >> 5, l = t & 31;
    if (4 * l >= tile_rows) return;
    // column j of the 4 x 4 block (row 4l + j) holds k = 4w .. 4w+3
    float4 col[4];
    col[0] = make_float4(v[0].x, v[1].x, v[2].x, v[3].x);
    col[1] = make_float4(v[0].y, v[1].y, v[2].y, v[3].y);
    col[2] = make_float4(v[0].z, v[1].z, v[2].z, v[3].z);
    col[3] = make_float4(v[0].w, v[1].w, v[2].w, v[3].w);
    const int rot = (l >> 1) & 3;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int jj = (j + rot) & 3;
      const float4 c = jj == 0 ? col[0] : jj == 1 ? col[1] : jj == 2 ? col[2] : col[3];
      st_split(hi, lo, tile_off(4 * l + jj, w), c);
    }
  }
};

// ---- epilogues ----------------------------------------------------------------
// A thread owns one accumulator row m and receives it in chunks of 16
// consecutive columns: begin(m), chunk(m, n0, v) for each of its chunks,
// end(m, key) (key = a per-thread index unique within the CTA tile).
struct EpiTanhBias {  // out[m, n] = tanh(acc + bias[n])
  float* out;
  const float* bias;
  int ld, M, N;
  __device__ __forceinline__ void begin(int) {}
  __device__ __forceinline__ void chunk(int m, int n0, const float (&v)[16]) {
    if (m >= M) return;
    float* o = out + (int64_t)m * ld;
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (n0 + i < N) o[n0 + i] = tanhf(v[i] + bias[n0 + i]);
  }
  __device__ __forceinline__ void end(int, int) {}
};

// h[m, n] = tanh(acc + b1[n]), plus the logits' partial sums over the
// thread's hidden units: zpart[part, m, c] = sum_n h[m, n] w2[n, c]
// (c < n_o <= NO), part = n_tile * 2 + key.
template <int NO>
struct EpiTanhLogits {
  float* out;
  const float* bias;
  const float* w2;
  float* zpart;
  int ld, M, N, n_o;
  float zp[NO];
  __device__ __forceinline__ void begin(int) {
#pragma unroll
    for (int c = 0; c < NO; ++c) zp[c] = 0.f;
  }
  __device__ __forceinline__ void chunk(int m, int n0, const float (&v)[16]) {
    if (m >= M) return;
    float* o = out + (int64_t)m * ld;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (n0 + i < N) {
        const float hv = tanhf(v[i] + bias[n0 + i]);
        o[n0 + i] = hv;
        const float* wr = w2 + (int64_t)(n0 + i) * n_o;  // same address across the warp
#pragma unroll
        for (int c = 0; c < NO; ++c)
          if (c < n_o) zp[c] = fmaf(hv, __ldg(wr + c), zp[c]);
      }
    }
  }
  __device__ __forceinline__ void end(int m, int key) {
    if (m >= M) return;
    float* zr = zpart + ((int64_t)(blockIdx.x * 2 + key) * M + m) * n_o;
#pragma unroll
    for (int c = 0; c < NO; ++c)
      if (c < n_o) zr[c] = zp[c];
  }
};

struct EpiAccumulate {  // out[m, n] += acc
  float* out;
  int ld, M, N;
  __device__ __forceinline__ void begin(int) {}
  __device__ __forceinline__ void chunk(int m, int n0, const float (&v)[16]) {
    if (m >= M) return;
    float* o = out + (int64_t)m * ld;
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (n0 + i < N) o[n0 + i] = o[n0 + i] + v[i];
  }
  __device__ __forceinline__ void end(int, int) {}
};

struct EpiPartial {  // part[slice, m, n] = acc (split-K slice of the contraction)
  float* part;
  int M, N;
  __device__ __forceinline__ void begin(int) {}
  __device__ __forceinline__ void chunk(int m, int n0, const float (&v)[16]) {
    if (m >= M) return;
    float* o = part + ((int64_t)blockIdx.z * M + m) * N;
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (n0 + i < N) o[n0 + i] = v[i];
  }
  __device__ __forceinline__ void end(int, int) {}
};

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// One CTA = one BM x BN output tile over one K slice. BN is a multiple of 16
// (<= 128); the B tile has BN rows.
template <int BN_, class LA, class LB, class EPI>
__global__ void __launch_bounds__(kThreads, 1)
tc_gemm_kernel(int M, int N, int K, int k_slice, LA la, LB lb, EPI epi) {
  static_assert(BN_ % 16 == 0 && BN_ >= 16 && BN_ <= 128, "tile width");
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw & 1023u)) & 1023u;
  uint8_t* tiles = smem_raw + pad;
  uint64_t* bars = reinterpret_cast<uint64_t*>(tiles + STAGES * kStageBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 1);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES);
  const uint32_t accb = smem_u32(bars + 2 * STAGES);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN_;
  const int kbeg = blockIdx.z * k_slice;
  const int kend = min(K, kbeg + k_slice);
  const int nkb = kend > kbeg ? (kend - kbeg + BK - 1) / BK : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, kXWarps * 32);
      mbar_init(empty0 + 8 * s, 1);
    }
    mbar_init(accb, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kMmaWarp) tmem_alloc(smem_u32(tmem_slot));
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp < kXWarps) {
    // ---- transform producers: loads run two K blocks ahead of the stores --------
    const int t = threadIdx.x;
    float4 va[2][4], vb[2][4];
    if (nkb > 0) {
      la.load(m0, kbeg, t, BM, va[0]);
      lb.load(n0, kbeg, t, BN_, vb[0]);
    }
    if (nkb > 1) {
      la.load(m0, kbeg + BK, t, BM, va[1]);
      lb.load(n0, kbeg + BK, t, BN_, vb[1]);
    }
    auto stage_out = [&](int kb, float4 (&a)[4], float4 (&b)[4]) -> bool {
      const int s = kb % STAGES;
      const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
      if (!mbar_wait(empty0 + 8 * s, ph ^ 1u)) return false;
      uint8_t* st = tiles + s * kStageBytes;
      la.store(st, st + kTileBytes, t, BM, a);
      lb.store(st + 2 * kTileBytes, st + 3 * kTileBytes, t, BN_, b);
      fence_proxy_async();
      mbar_arrive(full0 + 8 * s);
      if (kb + 2 < nkb) {
        const int k0 = kbeg + (kb + 2) * BK;
        la.load(m0, k0, t, BM, a);
        lb.load(n0, k0, t, BN_, b);
      }
      return true;
    };
    for (int kb = 0; kb < nkb && ok; kb += 2) {
      ok = stage_out(kb, va[0], vb[0]);
      if (ok && kb + 1 < nkb) ok = stage_out(kb + 1, va[1], vb[1]);
    }
    // ---- epilogue: TMEM -> registers -> global --------------------------------
    if (ok) ok = mbar_wait(accb, 0);
    tc_fence_after();
    // tcgen05.ld is warp-collective: the whole warp takes the same branch
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      const int quad = warp & 3, half = warp >> 2;
      const int m = m0 + quad * 32 + lane;
      epi.begin(m);
      for (int c = half; c < BN_ / 16; c += 2) {
        float v[16];
        tmem_ld16(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(c * 16), v);
        if (nkb == 0) {
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = 0.f;
        }
        epi.chunk(m, n0 + c * 16, v);
      }
      epi.end(m, half);
    }
  } else if (lane == 0) {
    // ---- MMA issuer -------------------------------------------------------------
    constexpr uint32_t idesc = idesc_tf32(BM, BN_);
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % STAGES;
      const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
      if (!mbar_wait(full0 + 8 * s, ph)) { ok = false; break; }
      tc_fence_after();
      const uint32_t st = smem_u32(tiles + s * kStageBytes);
#pragma unroll
      for (int j = 0; j < BK / 8; ++j) {
        const uint64_t ahi = desc_sw128(st + 32 * j);
        const uint64_t alo = desc_sw128(st + kTileBytes + 32 * j);
        const uint64_t bhi = desc_sw128(st + 2 * kTileBytes + 32 * j);
        const uint64_t blo = desc_sw128(st + 3 * kTileBytes + 32 * j);
        mma_tf32(tmem, ahi, blo, idesc, (kb | j) != 0 ? 1u : 0u);
        mma_tf32(tmem, alo, bhi, idesc, 1u);
        mma_tf32(tmem, ahi, bhi, idesc, 1u);
      }
      mma_commit(empty0 + 8 * s);
    }
    // arrives once every MMA issued above has completed (immediately if none)
    mma_commit(accb);
  }

  // ---- teardown: no tensor-core work may be in flight when TMEM is freed ----------
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    if (lane == 0) mbar_wait(accb, 0);
    __syncwarp();
    tmem_dealloc(tmem);
  }
}

// Sums split-K slices in slice order; rows < n_w go to w (accumulate), row
// n_w (the row of ones) to bias.
__global__ void tc_splitk_finish_kernel(const float* __restrict__ part, int splits, int M, int N,
                                        int n_w, float* __restrict__ w, float* __restrict__ bias) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t MN = (int64_t)M * N;
  if (e >= MN) return;
  float acc = 0.f;
  acc = ordered_sum(part + e, splits, MN);
  const int m = (int)(e / N), n = (int)(e % N);
  if (m < n_w) w[(int64_t)m * N + n] += acc;
  else bias[n] += acc;
}

struct Slices {
  int k_slice, count;
};
// K slices of at least 16 K blocks, the count chosen so that tiles x slices
// fills whole waves of one CTA per SM as nearly as possible.
inline Slices slices_for(int tiles, int K, int max_slices) {
  const int kblocks = (K + BK - 1) / BK;
  int best = 1;
  double best_eff = 0.0;
  for (int sl = 1; sl <= max_slices; ++sl) {
    if (sl > 1 && kblocks / sl < 16) break;
    const int ctas = tiles * sl;
    const int waves = (ctas + 147) / 148;
    const double eff = (double)ctas / (waves * 148.0);
    if (eff > best_eff + 1e-9 || (waves < 3 && sl > best)) {
      best_eff = eff;
      best = sl;
    }
    if (eff > 0.97 && waves >= 3) break;
  }
  const int per = (kblocks + best - 1) / best;
  Slices r;
  r.k_slice = (per > 0 ? per : 1) * BK;
  r.count = K > 0 ? (K + r.k_slice - 1) / r.k_slice : 1;
  return r;
}

template <int BN_, class LA, class LB, class EPI>
stade_status launch(int M, int N, int K, Slices sl, const LA& la, const LB& lb, const EPI& epi,
                    cudaStream_t s) {
  STADE_CUDA(cudaFuncSetAttribute(tc_gemm_kernel<BN_, LA, LB, EPI>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
  dim3 grid((N + BN_ - 1) / BN_, (M + BM - 1) / BM, sl.count);
  tc_gemm_kernel<BN_, LA, LB, EPI><<<grid, kThreads, kSmemBytes, s>>>(M, N, K, sl.k_slice, la, lb,
                                                                     epi);
  STADE_CHECK_LAUNCH();
  return STADE_OK;
}

inline Slices whole_k(int K) {
  Slices r;
  r.k_slice = (K > 0 ? (K + BK - 1) / BK : 1) * BK;
  r.count = 1;
  return r;
}

inline Slices w1b_slices(int S, int I, int H) {
  const int tiles = ((I + 1 + BM - 1) / BM) * ((H + BN - 1) / BN);
  return slices_for(tiles, S, 64);
}

}  // namespace tc

bool tc_mlp_supported(int64_t n_s, int64_t n_i, int64_t n_h) {
  return n_s >= 1 && n_i >= 1 && n_h >= 1 && n_i % 4 == 0 && n_h % 4 == 0 &&
         n_s < (int64_t(1) << 30) && n_i < (1 << 20) && n_h < (1 << 20);
}

size_t tc_mlp_workspace(int64_t n_s, int64_t n_i, int64_t n_h) {
  if (!tc_mlp_supported(n_s, n_i, n_h)) return 0;
  const int sp = tc::w1b_slices((int)n_s, (int)n_i, (int)n_h).count;
  return align_up((size_t)sp * (size_t)(n_i + 1) * (size_t)n_h * sizeof(float), 256);
}

int tc_logit_parts(int64_t n_h) { return 2 * (int)((n_h + tc::BN - 1) / tc::BN); }

stade_status tc_forward_tanh(const float* x, const float* w1, const float* b1, float* h, int S,
                             int I, int H, void*, cudaStream_t s) {
  // A[m = sample, k = input] = x (K-contiguous); B[n = hidden, k = input] = w1[k, n]
  tc::LoadK la{x, I, S, I, -1};
  tc::LoadMN lb{w1, H, H, I, -1};
  tc::EpiTanhBias epi{h, b1, H, S, H};
  return tc::launch<tc::BN>(S, H, I, tc::whole_k(I), la, lb, epi, s);
}

stade_status tc_forward_tanh_logits(const float* x, const float* w1, const float* b1,
                                    const float* w2, float* h, float* zpart, int S, int I, int H,
                                    int O, cudaStream_t s) {
  tc::LoadK la{x, I, S, I, -1};
  tc::LoadMN lb{w1, H, H, I, -1};
  if (O <= 16)
    return tc::launch<tc::BN>(S, H, I, tc::whole_k(I), la, lb,
                              tc::EpiTanhLogits<16>{h, b1, w2, zpart, H, S, H, O, {}}, s);
  return tc::launch<tc::BN>(S, H, I, tc::whole_k(I), la, lb,
                            tc::EpiTanhLogits<32>{h, b1, w2, zpart, H, S, H, O, {}}, s);
}

stade_status tc_weight_grad(const float* x, const float* s1b, float* w1b, float* b1b, int S, int I,
                            int H, void* ws, cudaStream_t s) {
  // A[m = input (+ row of ones), k = sample] = x[k, m]; B[n = hidden, k = sample] = s1b[k, n]
  const int M = I + 1;
  const tc::Slices sl = tc::w1b_slices(S, I, H);
  float* part = static_cast<float*>(ws);
  tc::LoadMN la{x, I, I, S, I};
  tc::LoadMN lb{s1b, H, H, S, -1};
  tc::EpiPartial epi{part, M, H};
  stade_status st = tc::launch<tc::BN>(M, H, S, sl, la, lb, epi, s);
  if (st != STADE_OK) return st;
  const int64_t MN = (int64_t)M * H;
  tc::tc_splitk_finish_kernel<<<ceil_div_u(MN, 256), 256, 0, s>>>(part, sl.count, M, H, I, w1b,
                                                                   b1b);
  STADE_CHECK_LAUNCH();
  return STADE_OK;
}

stade_status tc_input_grad(const float* s1b, const float* w1, float* xb, int S, int I, int H, void*,
                           cudaStream_t s) {
  // A[m = sample, k = hidden] = s1b (K-contiguous); B[n = input, k = hidden] = w1[n, k].
  // The tile width divides the input width when it can (784 = 7 x 112).
  tc::LoadK la{s1b, H, S, H, -1};
  tc::LoadK lb{w1, H, I, H, -1};
  tc::EpiAccumulate epi{xb, I, S, I};
  if (I % 128 != 0 && I % 112 == 0)
    return tc::launch<112>(S, I, H, tc::whole_k(H), la, lb, epi, s);
  if (I % 128 != 0 && I % 96 == 0)
    return tc::launch<96>(S, I, H, tc::whole_k(H), la, lb, epi, s);
  return tc::launch<tc::BN>(S, I, H, tc::whole_k(H), la, lb, epi, s);
}

}  // namespace stade

namespace stade {
int tma_take_error();
int conv_tc_take_error();
}

extern "C" int stade_device_error(void) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, stade::tc::g_tc_error, sizeof(int)) != cudaSuccess) return -1;
  if (v) {
    const int zero = 0;
    cudaMemcpyToSymbol(stade::tc::g_tc_error, &zero, sizeof(int));
  }
  const int t = stade::tma_take_error();
  const int c = stade::conv_tc_take_error();
  if (t < 0 || c < 0) return -1;
  return v | t | c;
}
