// gdn_prefill.cu — GDN chunked prefill on the sm_100a tensor cores (tcgen05).
//
// The reference defines prefill only as T applications of its decode
// recurrence (pytorch_reference_gdn.py:38-91; chunking is described, not
// implemented, in analysis/wave15-attention-research/MECHANISMS.md:398-445).
// This kernel computes the same result chunk by chunk (chunk C = 64 tokens).
// Per chunk, with G the in-chunk cumulative log gate, gamma = exp(G):
//   A[i][j] = beta_i exp(G_i - G_j) k_i.k_j            (j < i)
//   T       = (I + A)^-1                                (blocked forward substitution, fp32)
//   W       = T diag(beta gamma) K,   U = T diag(beta) V
//   V'      = U - W S                                   (S: state entering the chunk)
//   O       = diag(gamma) Q S + (Q K^T . causal . exp(G_i - G_j)) V'
//   S_next  = gamma_C S + K^T diag(exp(G_C - G_j)) V'
// which unrolls the recurrence S_t = a_t S_{t-1} + beta_t k_t (v_t - a_t S_{t-1}^T k_t)^T
// exactly (in exact arithmetic).
//
// Every product is a tcgen05.mma with M = 128, written transposed so the 128
// TMEM lanes index d_v (or d_k): [K;Q] K^T, W^T = K^T T_w^T, U^T = V^T T_u^T,
// X^T = S^T W^T, Z^T = S^T Q^T, O_intra^T = V'^T P^T, dS^T = V''^T K.
// Operands are bf16 (f16) in 128B-swizzled shared memory; TMA fills the
// K/Q/V tiles and the same tile serves as K-major and MN-major operand.
// Accumulators live in TMEM (512 columns); the fp32 master state lives in
// registers (thread = one d_v row of S^T, 64 of its d_k columns).
// Precision: the decayed V'' = diag(exp(G_C - G_j)) V' that updates the state
// is split into bf16 hi + lo halves (two MMAs), and K enters the state update
// unscaled, so the state accumulates with ~16 mantissa bits per term.
//
// One CTA per (batch, value head), 256 threads (8 warps).  Warp w reads TMEM
// lane quarter w % 4; warps w and w + 4 split the columns.
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "ptx.cuh"
#include "tc.cuh"

namespace gdn {
namespace prefill {

#ifdef GDN_PREFILL_TRACE
// Phase timestamps of CTA 0 (profiling builds only): [chunk][phase].
__device__ unsigned long long g_trace[64 * 12];
#define TRACE(c, ph)                                                              \
  do {                                                                            \
    if (blockIdx.x == 0 && threadIdx.x == 0 && (c) < 64) g_trace[(c) * 12 + (ph)] = \
        global_timer_ns();                                                        \
  } while (0)
#else
#define TRACE(c, ph) \
  do {               \
  } while (0)
#endif

constexpr int kC = 64;     // chunk length
constexpr int kD = 128;    // d_k = d_v
constexpr int kThreads = 256;

// shared-memory map (byte offsets from a 1024-aligned base)
constexpr uint32_t kKQ = 0;            // 2 buffers x [K | Q] tile: 2 d_k blocks x (K 8 KB + Q 8 KB)
constexpr uint32_t kKQBuf = 32768;
constexpr uint32_t kKQBlock = 16384;
constexpr uint32_t kV = 65536;         // 2 buffers x V tile: 2 d_v blocks x 8 KB
constexpr uint32_t kVBuf = 16384;
constexpr uint32_t kVBlock = 8192;
constexpr uint32_t kTw = 98304;        // T diag(beta gamma), K-major rows i   (8 KB)
constexpr uint32_t kTu = 106496;       // T diag(beta), K-major rows i          (8 KB)
constexpr uint32_t kP = 114688;        // causal decayed QK^T, rows i           (8 KB)
constexpr uint32_t kWT = 122880;       // W^T, MN-major rows d_k               (16 KB)
constexpr uint32_t kST = 139264;       // S^T bf16, K-major rows d_v, 2 blocks (32 KB)
constexpr uint32_t kSTBlock = 16384;
constexpr uint32_t kVP = 172032;       // V'^T, K-major rows d_v               (16 KB)
constexpr uint32_t kVH = 188416;       // V''^T hi                             (16 KB)
constexpr uint32_t kVL = 204800;       // V''^T lo                             (16 KB)
// fp32 solver matrices (row stride 68 floats) alias V'/V''hi/V''lo, which are
// dead between the previous chunk's last MMA and this chunk's epilogue.
constexpr int kLd = 68;
constexpr uint32_t kAf = kVP;                       // A   [64][68]
constexpr uint32_t kTf = kVP + 64 * kLd * 4;        // T   [64][68]
constexpr uint32_t kMs = kVP + 2 * 64 * kLd * 4;    // merge scratch (32 x 68 floats)
constexpr uint32_t kVec = 221184;      // 4 x 64 fp32: G, gamma, beta, raw g
constexpr uint32_t kBars = kVec + 1024;
constexpr uint32_t kSmemBytes = kBars + 64;
constexpr uint32_t kSmemAlloc = kSmemBytes + 1024;  // + alignment slack
static_assert(kMs + 32 * kLd * 4 <= kVL + 16384, "solver scratch overflows its alias");

// TMEM columns
constexpr uint32_t kTmKQ = 0, kTmZ = 64, kTmW = 128, kTmU = 192, kTmX = 256, kTmOI = 320,
                   kTmDS = 384, kTmCols = 512;

struct Params {
  gdn_prefill_args_t a;
  int32_t nchunks;
  int32_t group;
};

template <bool BF16>
__device__ __forceinline__ void store_row16(uint32_t tile, int row, int chunk0, const float* v) {
  tc::sts128(tile + tc::sw128_offset(row, chunk0), tc::pack2<BF16>(v[0], v[1]),
             tc::pack2<BF16>(v[2], v[3]), tc::pack2<BF16>(v[4], v[5]), tc::pack2<BF16>(v[6], v[7]));
  tc::sts128(tile + tc::sw128_offset(row, chunk0 + 1), tc::pack2<BF16>(v[8], v[9]),
             tc::pack2<BF16>(v[10], v[11]), tc::pack2<BF16>(v[12], v[13]),
             tc::pack2<BF16>(v[14], v[15]));
}

// Every thread waits (bounded) on the barrier phase; the CTA then agrees on
// the outcome, so a timeout unwinds all threads together.
__device__ __forceinline__ bool cta_wait(uint64_t* bar, uint32_t parity) {
  const bool ok = mbar_wait_bounded(bar, parity);
  return __syncthreads_and(ok) != 0;
}

// ------------------------------------------------------------ triangular solve
// m16n8k8 TF32 warp MMA with the 3xTF32 split (hi*hi + hi*lo + lo*hi), which
// keeps the block products of the solve at close to fp32 accuracy.
__device__ __forceinline__ void tf32_split(float x, uint32_t& hi, uint32_t& lo) {
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(hi) : "f"(x));
  const float r = x - __uint_as_float(hi);
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(lo) : "f"(r));
}

__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// acc (16 x 16, two m16n8 fragments) += X (16 x 16 block at x, stride kLd) * Y (16 x 16 at y).
__device__ __forceinline__ void block_mma(float (&acc)[2][4], const float* x, const float* y, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int ks = 0; ks < 2; ++ks) {
    uint32_t ah[4], al[4];
    tf32_split(x[g * kLd + ks * 8 + t], ah[0], al[0]);
    tf32_split(x[(g + 8) * kLd + ks * 8 + t], ah[1], al[1]);
    tf32_split(x[g * kLd + ks * 8 + t + 4], ah[2], al[2]);
    tf32_split(x[(g + 8) * kLd + ks * 8 + t + 4], ah[3], al[3]);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      uint32_t bh[2], bl[2];
      tf32_split(y[(ks * 8 + t) * kLd + nt * 8 + g], bh[0], bl[0]);
      tf32_split(y[(ks * 8 + t + 4) * kLd + nt * 8 + g], bh[1], bl[1]);
      mma_tf32(acc[nt], al, bh);
      mma_tf32(acc[nt], ah, bl);
      mma_tf32(acc[nt], ah, bh);
    }
  }
}

__device__ __forceinline__ void block_store(float* z, const float (&acc)[2][4], float sign, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    *reinterpret_cast<float2*>(z + g * kLd + nt * 8 + 2 * t) = make_float2(sign * acc[nt][0], sign * acc[nt][1]);
    *reinterpret_cast<float2*>(z + (g + 8) * kLd + nt * 8 + 2 * t) =
        make_float2(sign * acc[nt][2], sign * acc[nt][3]);
  }
}

// T = (I + A)^-1 for strictly lower-triangular A (64 x 64 fp32, stride kLd).
// 1) the four 16 x 16 diagonal blocks D_r by forward substitution (one warp
//    per block, one lane per column, fp32);  2) T_10 = -D_1 A_10 D_0 and
// T_32 = -D_3 A_32 D_2;  3) the lower-left 32 x 32 quadrant
// -T_bot A_bl T_top.  The block products run on m16n8k8 TF32 warp MMAs.
// Only the lower triangle of T is written.
__device__ __forceinline__ void solve_unit_lower(const float* A, float* T, float* M, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  if (warp < 4) {
    if (lane < 16) {
      const int bb = warp * 16, c = lane;
      float t[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) t[i] = (i == c) ? 1.f : 0.f;
#pragma unroll
      for (int i = 1; i < 16; ++i) {
        const float* row = A + (bb + i) * kLd + bb;
        float acc = 0.f;
#pragma unroll
        for (int j4 = 0; j4 < i; j4 += 4) {
          const float4 a4 = *reinterpret_cast<const float4*>(row + j4);
          acc = fmaf(a4.x, t[j4], acc);
          if (j4 + 1 < i) acc = fmaf(a4.y, t[j4 + 1], acc);
          if (j4 + 2 < i) acc = fmaf(a4.z, t[j4 + 2], acc);
          if (j4 + 3 < i) acc = fmaf(a4.w, t[j4 + 3], acc);
        }
        t[i] -= acc;
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) T[(bb + i) * kLd + bb + c] = t[i];
    }
  }
  __syncthreads();
  // level 1: warps 0 and 1 build T_10 and T_32 (X = A_rc D_c in scratch, then -D_r X)
  if (warp < 2) {
    const int c = warp * 2, r = c + 1;
    float* X = M + warp * 16 * kLd;
    float acc[2][4] = {};
    block_mma(acc, A + 16 * r * kLd + 16 * c, T + 16 * c * kLd + 16 * c, lane);
    block_store(X, acc, 1.f, lane);
    __syncwarp();
    float acc2[2][4] = {};
    block_mma(acc2, T + 16 * r * kLd + 16 * r, X, lane);
    block_store(T + 16 * r * kLd + 16 * c, acc2, -1.f, lane);
  }
  __syncthreads();
  // level 2: warp (r-2)*2 + c builds Y_rc = sum_k A_rk T_kc over the top blocks
  if (warp < 4) {
    const int r = 2 + (warp >> 1), c = warp & 1;
    float acc[2][4] = {};
    if (c == 0) {
      block_mma(acc, A + 16 * r * kLd + 0, T + 0, lane);                         // A_r0 D_0
      block_mma(acc, A + 16 * r * kLd + 16, T + 16 * kLd + 0, lane);             // A_r1 T_10
    } else {
      block_mma(acc, A + 16 * r * kLd + 16, T + 16 * kLd + 16, lane);            // A_r1 D_1
    }
    block_store(M + (r - 2) * 16 * kLd + 16 * c, acc, 1.f, lane);
  }
  __syncthreads();
  if (warp < 4) {
    const int r = 2 + (warp >> 1), c = warp & 1;
    float acc[2][4] = {};
    if (r == 2) {
      block_mma(acc, T + 32 * kLd + 32, M + 16 * c, lane);                       // D_2 Y_2c
    } else {
      block_mma(acc, T + 48 * kLd + 32, M + 16 * c, lane);                       // T_32 Y_2c
      block_mma(acc, T + 48 * kLd + 48, M + 16 * kLd + 16 * c, lane);            // D_3 Y_3c
    }
    block_store(T + 16 * r * kLd + 16 * c, acc, -1.f, lane);
  }
  __syncthreads();
}

template <bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const Params p, const __grid_constant__ CUtensorMap map_q,
                   const __grid_constant__ CUtensorMap map_k,
                   const __grid_constant__ CUtensorMap map_v) {
  using IO = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  float* sG = reinterpret_cast<float*>(smem + kVec);
  float* sGam = sG + 64;
  float* sBeta = sG + 128;
  float* sGraw = sG + 192;
  float* Af = reinterpret_cast<float*>(smem + kAf);
  float* Tf = reinterpret_cast<float*>(smem + kTf);
  float* Ms = reinterpret_cast<float*>(smem + kMs);
  uint64_t* tma_bar = reinterpret_cast<uint64_t*>(smem + kBars);  // [2]
  uint64_t* mma_bar = tma_bar + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tma_bar + 3);

  const gdn_prefill_args_t& a = p.a;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, half = warp >> 2;
  const int bh = blockIdx.x;
  const int b = bh / a.Hv, h = bh % a.Hv, hq = h / p.group;
  const int T = a.T;

  if (warp == 0) tc::tmem_alloc(tmem_holder, kTmCols);
  if (tid == 0) {
    mbar_init(&tma_bar[0], 1);
    mbar_init(&tma_bar[1], 1);
    mbar_init(mma_bar, 1);
    fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_holder;
  const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
  constexpr uint32_t kIdKQ = tc::idesc_f16(128, 64, false, false, BF16);
  constexpr uint32_t kIdW = tc::idesc_f16(128, 64, true, false, BF16);
  constexpr uint32_t kIdX = tc::idesc_f16(128, 64, false, true, BF16);
  constexpr uint32_t kIdDS = tc::idesc_f16(128, 128, false, true, BF16);

  // ---- master state: thread owns S[k][dv] for k in [k0, k0 + 64)
  const int dv = quarter * 32 + lane;
  const int k0 = half * 64;
  const size_t state_off = static_cast<size_t>(bh) * kD * kD;
  float S[64];
#pragma unroll
  for (int j = 0; j < 64; ++j)
    S[j] = a.initial_state ? a.initial_state[state_off + static_cast<size_t>(k0 + j) * kD + dv] : 0.f;
#pragma unroll
  for (int cc = 0; cc < 8; ++cc) {
    tc::sts128(sb + kST + half * kSTBlock + tc::sw128_offset(dv, cc),
               tc::pack2<BF16>(S[8 * cc + 0], S[8 * cc + 1]), tc::pack2<BF16>(S[8 * cc + 2], S[8 * cc + 3]),
               tc::pack2<BF16>(S[8 * cc + 4], S[8 * cc + 5]), tc::pack2<BF16>(S[8 * cc + 6], S[8 * cc + 7]));
  }
  tc::fence_proxy_async();

  auto issue_tma = [&](int chunk) {
    const int t0 = chunk * kC, buf = chunk & 1;
    uint64_t* bar = &tma_bar[buf];
    mbar_arrive_expect_tx(bar, 6 * 8192);
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
      unsigned char* kq = smem + kKQ + buf * kKQBuf + blk * kKQBlock;
      tc::tma_load_4d(kq, &map_k, blk * 64, hq, t0, b, bar);
      tc::tma_load_4d(kq + 8192, &map_q, blk * 64, hq, t0, b, bar);
      tc::tma_load_4d(smem + kV + buf * kVBuf + blk * kVBlock, &map_v, blk * 64, h, t0, b, bar);
    }
  };
  if (tid == 0) issue_tma(0);

  // gates of the next chunk are prefetched one chunk ahead into registers
  float g_next = 0.f, b_next = 0.f;
  auto load_gates = [&](int chunk) {
    const int t = chunk * kC + tid;
    if (tid < kC && t < T) {
      const int64_t gi = (static_cast<int64_t>(b) * T + t) * a.Hv + h;
      g_next = load_any(a.g, gi, a.g_dtype);
      b_next = load_any(a.beta, gi, a.beta_dtype);
    } else {
      g_next = 0.f;
      b_next = 0.f;
    }
  };
  load_gates(0);
  uint32_t mma_phase = 0;
  bool failed = false;

#pragma unroll 1
  for (int c = 0; c < p.nchunks; ++c) {
    const int t0 = c * kC, buf = c & 1;
    const uint32_t kq = sb + kKQ + buf * kKQBuf;
    const uint32_t vt = sb + kV + buf * kVBuf;
    if (tid < kC) {
      sGraw[tid] = g_next;
      sBeta[tid] = b_next;
    }
    if (!cta_wait(&tma_bar[buf], (c >> 1) & 1)) { failed = true; break; }
    TRACE(c, 0);
    if (tid == 0 && c + 1 < p.nchunks) issue_tma(c + 1);  // into the other buffer
    if (c + 1 < p.nchunks) load_gates(c + 1);

    // ---- MMA 1: [K;Q] K^T -> KQ ; S^T Q^T -> Z
    if (tid == 0) {
      tc::fence_after_sync();
#pragma unroll
      for (int s = 0; s < 8; ++s)
        tc::mma(tmem + kTmKQ, tc::kmajor_desc(kq, kKQBlock, s), tc::kmajor_desc(kq, kKQBlock, s), kIdKQ,
                s > 0);
#pragma unroll
      for (int s = 0; s < 8; ++s)
        tc::mma(tmem + kTmZ, tc::kmajor_desc(sb + kST, kSTBlock, s),
                tc::kmajor_desc(kq + 8192, kKQBlock, s), kIdKQ, s > 0);
      tc::commit(mma_bar);
    }
    // ---- in-chunk cumulative gate (warp 0): lane l owns tokens 2l, 2l+1
    if (warp == 0) {
      const float g0 = sGraw[2 * lane], g1 = sGraw[2 * lane + 1];
      float run = g0 + g1;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float o = __shfl_up_sync(0xffffffffu, run, off);
        if (lane >= off) run += o;
      }
      const float excl = run - (g0 + g1);
      sG[2 * lane] = excl + g0;
      sG[2 * lane + 1] = run;
      sGam[2 * lane] = __expf(excl + g0);
      sGam[2 * lane + 1] = __expf(run);
    }
    if (!cta_wait(mma_bar, mma_phase)) { failed = true; break; }
    mma_phase ^= 1;
    tc::fence_after_sync();
    TRACE(c, 1);

    // ---- A rows (K K^T, TMEM lanes 0-63) and P rows (Q K^T, lanes 64-127);
    //      warps w and w+4 take columns [0,32) and [32,64)
    {
      const int i = (quarter & 1) * 32 + lane;
      const float Gi = sG[i];
      float r[32];
      tc::tmem_ld16(tmem + lane_base + kTmKQ + half * 32, *reinterpret_cast<float(*)[16]>(r));
      tc::tmem_ld16(tmem + lane_base + kTmKQ + half * 32 + 16, *reinterpret_cast<float(*)[16]>(r + 16));
      tc::tmem_wait_ld();
      if (quarter < 2) {
        const float bi = sBeta[i];
#pragma unroll
        for (int j4 = 0; j4 < 32; j4 += 4) {
          float4 v;
          float* pv = reinterpret_cast<float*>(&v);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = half * 32 + j4 + e;
            pv[e] = (j < i) ? bi * __expf(Gi - sG[j]) * r[j4 + e] : 0.f;
          }
          *reinterpret_cast<float4*>(Af + i * kLd + half * 32 + j4) = v;
        }
      } else {
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int j = half * 32 + jj;
          r[jj] = (j <= i) ? r[jj] * __expf(Gi - sG[j]) : 0.f;
        }
        store_row16<BF16>(sb + kP, i, half * 4, r);
        store_row16<BF16>(sb + kP, i, half * 4 + 2, r + 16);
      }
    }
    __syncthreads();
    TRACE(c, 2);
    solve_unit_lower(Af, Tf, Ms, tid);
    TRACE(c, 3);
    {
      const int i = tid >> 2, jq = tid & 3;
      float tw[16], tu[16];
#pragma unroll
      for (int j4 = 0; j4 < 16; j4 += 4) {
        const float4 t4 = *reinterpret_cast<const float4*>(Tf + i * kLd + jq * 16 + j4);
        const float tv[4] = {t4.x, t4.y, t4.z, t4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j = jq * 16 + j4 + e;
          const float t = (j <= i) ? tv[e] : 0.f;
          tu[j4 + e] = t * sBeta[j];
          tw[j4 + e] = tu[j4 + e] * sGam[j];
        }
      }
      store_row16<BF16>(sb + kTw, i, jq * 2, tw);
      store_row16<BF16>(sb + kTu, i, jq * 2, tu);
    }
    tc::fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    TRACE(c, 4);

    // ---- MMA 2: W^T = K^T T_w^T ; U^T = V^T T_u^T
    if (tid == 0) {
      tc::fence_after_sync();
#pragma unroll
      for (int s = 0; s < 4; ++s)
        tc::mma(tmem + kTmW, tc::mnmajor_desc(kq, kKQBlock, s), tc::kmajor_desc(sb + kTw, 0, s), kIdW,
                s > 0);
#pragma unroll
      for (int s = 0; s < 4; ++s)
        tc::mma(tmem + kTmU, tc::mnmajor_desc(vt, kVBlock, s), tc::kmajor_desc(sb + kTu, 0, s), kIdW,
                s > 0);
      tc::commit(mma_bar);
    }
    if (!cta_wait(mma_bar, mma_phase)) { failed = true; break; }
    mma_phase ^= 1;
    tc::fence_after_sync();
    TRACE(c, 5);
    {  // W^T -> bf16 tile, MN-major rows d_k = quarter*32 + lane, tokens [32 half, +32)
      const int k = quarter * 32 + lane;
      float r[32];
      tc::tmem_ld16(tmem + lane_base + kTmW + half * 32, *reinterpret_cast<float(*)[16]>(r));
      tc::tmem_ld16(tmem + lane_base + kTmW + half * 32 + 16, *reinterpret_cast<float(*)[16]>(r + 16));
      tc::tmem_wait_ld();
      store_row16<BF16>(sb + kWT, k, half * 4, r);
      store_row16<BF16>(sb + kWT, k, half * 4 + 2, r + 16);
    }
    tc::fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    TRACE(c, 6);

    // ---- MMA 3: X^T = S^T W^T
    if (tid == 0) {
      tc::fence_after_sync();
#pragma unroll
      for (int s = 0; s < 8; ++s)
        tc::mma(tmem + kTmX, tc::kmajor_desc(sb + kST, kSTBlock, s), tc::mnmajor_desc(sb + kWT, 8192, s),
                kIdX, s > 0);
      tc::commit(mma_bar);
    }
    if (!cta_wait(mma_bar, mma_phase)) { failed = true; break; }
    mma_phase ^= 1;
    tc::fence_after_sync();
    TRACE(c, 7);
    {  // V' = U - X ; V'' = V' exp(G_C - G_j) split hi / lo
      const float GC = sG[kC - 1];
      float u[32], x[32];
      tc::tmem_ld16(tmem + lane_base + kTmU + half * 32, *reinterpret_cast<float(*)[16]>(u));
      tc::tmem_ld16(tmem + lane_base + kTmU + half * 32 + 16, *reinterpret_cast<float(*)[16]>(u + 16));
      tc::tmem_ld16(tmem + lane_base + kTmX + half * 32, *reinterpret_cast<float(*)[16]>(x));
      tc::tmem_ld16(tmem + lane_base + kTmX + half * 32 + 16, *reinterpret_cast<float(*)[16]>(x + 16));
      tc::tmem_wait_ld();
#pragma unroll
      for (int cb = 0; cb < 2; ++cb) {
        float vp[16], hi[16], lo[16];
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
          const int j = half * 32 + cb * 16 + jj;
          vp[jj] = u[cb * 16 + jj] - x[cb * 16 + jj];
          const float vd = vp[jj] * __expf(GC - sG[j]);
          hi[jj] = tc::unpack_lo<BF16>(tc::pack2<BF16>(vd, 0.f));
          lo[jj] = vd - hi[jj];
        }
        store_row16<BF16>(sb + kVP, dv, half * 4 + cb * 2, vp);
        store_row16<BF16>(sb + kVH, dv, half * 4 + cb * 2, hi);
        store_row16<BF16>(sb + kVL, dv, half * 4 + cb * 2, lo);
      }
    }
    tc::fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    TRACE(c, 8);

    // ---- MMA 4: O_intra^T = V'^T P^T ; dS^T = V''hi^T K + V''lo^T K
    if (tid == 0) {
      tc::fence_after_sync();
#pragma unroll
      for (int s = 0; s < 4; ++s)
        tc::mma(tmem + kTmOI, tc::kmajor_desc(sb + kVP, 0, s), tc::kmajor_desc(sb + kP, 0, s), kIdKQ,
                s > 0);
#pragma unroll
      for (int s = 0; s < 4; ++s)
        tc::mma(tmem + kTmDS, tc::kmajor_desc(sb + kVH, 0, s), tc::mnmajor_desc(kq, kKQBlock, s), kIdDS,
                s > 0);
#pragma unroll
      for (int s = 0; s < 4; ++s)
        tc::mma(tmem + kTmDS, tc::kmajor_desc(sb + kVL, 0, s), tc::mnmajor_desc(kq, kKQBlock, s), kIdDS,
                true);
      tc::commit(mma_bar);
    }
    if (!cta_wait(mma_bar, mma_phase)) { failed = true; break; }
    mma_phase ^= 1;
    tc::fence_after_sync();
    TRACE(c, 9);

    {  // state update and bf16 copy for the next chunk
      const float gC = sGam[kC - 1];
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        float r[32];
        tc::tmem_ld16(tmem + lane_base + kTmDS + half * 64 + hb * 32, *reinterpret_cast<float(*)[16]>(r));
        tc::tmem_ld16(tmem + lane_base + kTmDS + half * 64 + hb * 32 + 16,
                      *reinterpret_cast<float(*)[16]>(r + 16));
        tc::tmem_wait_ld();
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) S[hb * 32 + jj] = fmaf(gC, S[hb * 32 + jj], r[jj]);
      }
#pragma unroll
      for (int cc = 0; cc < 8; ++cc)
        tc::sts128(sb + kST + half * kSTBlock + tc::sw128_offset(dv, cc),
                   tc::pack2<BF16>(S[8 * cc + 0], S[8 * cc + 1]), tc::pack2<BF16>(S[8 * cc + 2], S[8 * cc + 3]),
                   tc::pack2<BF16>(S[8 * cc + 4], S[8 * cc + 5]), tc::pack2<BF16>(S[8 * cc + 6], S[8 * cc + 7]));
    }
    {  // outputs o[t0 + i][dv] = scale (gamma_i Z[dv][i] + O_intra[dv][i])
      IO* o = static_cast<IO*>(a.o);
      float z[32], oi[32];
      tc::tmem_ld16(tmem + lane_base + kTmZ + half * 32, *reinterpret_cast<float(*)[16]>(z));
      tc::tmem_ld16(tmem + lane_base + kTmZ + half * 32 + 16, *reinterpret_cast<float(*)[16]>(z + 16));
      tc::tmem_ld16(tmem + lane_base + kTmOI + half * 32, *reinterpret_cast<float(*)[16]>(oi));
      tc::tmem_ld16(tmem + lane_base + kTmOI + half * 32 + 16, *reinterpret_cast<float(*)[16]>(oi + 16));
      tc::tmem_wait_ld();
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        const int i = half * 32 + jj;
        const int t = t0 + i;
        if (t < T)
          o[((static_cast<int64_t>(b) * T + t) * a.Hv + h) * kD + dv] =
              from_f32<IO>(a.scale * fmaf(sGam[i], z[jj], oi[jj]));
      }
    }
    tc::fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    TRACE(c, 10);
  }

  if (failed) {
    if (tid == 0) report(a.status, GDN_DEVERR_MMA_TIMEOUT);
  } else {
#pragma unroll
    for (int j = 0; j < 64; ++j)
      a.final_state[state_off + static_cast<size_t>(k0 + j) * kD + dv] = S[j];
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, kTmCols);
}

template <bool BF16>
int launch(const gdn_prefill_args_t& a, cudaStream_t stream) {
  static std::atomic<uint64_t> attr_done{0};
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  if (static_cast<int>(kSmemAlloc) > di.smem_optin) return GDN_ERR_SHAPE;
  auto kern = prefill_kernel<BF16>;
  rc = ensure_smem_attr(kern, kSmemAlloc, attr_done);
  if (rc) return rc;
  const CUtensorMapDataType dt = BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap mq, mk, mv;
  const uint32_t box[4] = {64, 1, kC, 1};
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(a.dk), static_cast<uint64_t>(a.Hqk),
                              static_cast<uint64_t>(a.T), static_cast<uint64_t>(a.B)};
    const uint64_t str[3] = {static_cast<uint64_t>(a.dk) * 2, static_cast<uint64_t>(a.Hqk) * a.dk * 2,
                             static_cast<uint64_t>(a.T) * a.Hqk * a.dk * 2};
    if ((rc = tensor_map(&mq, dt, 4, a.q, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
    if ((rc = tensor_map(&mk, dt, 4, a.k, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  }
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(a.dv), static_cast<uint64_t>(a.Hv),
                              static_cast<uint64_t>(a.T), static_cast<uint64_t>(a.B)};
    const uint64_t str[3] = {static_cast<uint64_t>(a.dv) * 2, static_cast<uint64_t>(a.Hv) * a.dv * 2,
                             static_cast<uint64_t>(a.T) * a.Hv * a.dv * 2};
    if ((rc = tensor_map(&mv, dt, 4, a.v, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  }
  Params p;
  p.a = a;
  p.nchunks = (a.T + kC - 1) / kC;
  p.group = a.Hv / a.Hqk;
  kern<<<static_cast<unsigned>(a.B * a.Hv), kThreads, kSmemAlloc, stream>>>(p, mq, mk, mv);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

int validate(const gdn_prefill_args_t* a) {
  if (!a) return GDN_ERR_NULL;
  if (!a->q || !a->k || !a->v || !a->g || !a->beta || !a->final_state || !a->o) return GDN_ERR_NULL;
  if (a->B < 1 || a->T < 1 || a->Hqk < 1 || a->Hv < 1 || a->Hv % a->Hqk) return GDN_ERR_SHAPE;
  if (a->dk != kD || a->dv != kD || a->chunk != kC) return GDN_ERR_SHAPE;
  if (static_cast<int64_t>(a->B) * a->Hv > 0x7FFFFFFF) return GDN_ERR_SHAPE;
  if (a->io_dtype != GDN_DT_BF16 && a->io_dtype != GDN_DT_F16) return GDN_ERR_DTYPE;
  if (!dtype_valid(a->g_dtype) || !dtype_valid(a->beta_dtype)) return GDN_ERR_DTYPE;
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->o) ||
      !aligned16(a->final_state) || (a->initial_state && !aligned16(a->initial_state)))
    return GDN_ERR_ALIGN;
  return GDN_OK;
}

}  // namespace prefill
}  // namespace gdn

#ifdef GDN_PREFILL_TRACE
extern "C" int gdn_prefill_trace_read(unsigned long long* host) {
  return cudaMemcpyFromSymbol(host, gdn::prefill::g_trace, sizeof(gdn::prefill::g_trace)) ==
                 cudaSuccess
             ? 0
             : 1;
}
#endif

extern "C" size_t gdn_prefill_workspace_size(const gdn_prefill_args_t*) { return 0; }

extern "C" int gdn_prefill_launch(const gdn_prefill_args_t* args, gdn_stream_t stream) {
  int rc = gdn::prefill::validate(args);
  if (rc) return rc;
  gdn::DeviceInfo di;
  if ((rc = gdn::device_info(&di))) return rc;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  return args->io_dtype == GDN_DT_BF16 ? gdn::prefill::launch<true>(*args, s)
                                       : gdn::prefill::launch<false>(*args, s);
}
