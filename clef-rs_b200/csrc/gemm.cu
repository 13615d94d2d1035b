// gemm.cu — BF16 projection GEMM on the sm_100a tensor cores.
//
// Y[M, N] = X[M, K] * W[N, K]^T with F32 accumulation, the layout of every
// projection of the backbone (Projection::forward, projection.rs:82-95; the
// reference's Metal tile kernel, neural.metal:72-125).
//
// One persistent CTA per SM walks 128 x 256 output tiles in a grouped raster
// (8 N-tiles share each A row-block while it is hot in L2). Warp roles:
//   warp 0      TMA producer: A and B tiles (64-wide K slabs, 128-byte
//               swizzle) into a 4-stage shared-memory ring, no multicast;
//   warp 1      allocates 512 TMEM columns and, from one thread, issues
//               tcgen05.mma 128x256x16 into one of two TMEM accumulators;
//   warps 2..5  epilogue: tcgen05.ld the accumulator (each warp its 32-lane
//               quarter), apply the epilogue, store to global memory, then
//               release the accumulator so the next tile's MMAs overlap it.
// Epilogues: BF16 store, F32 store, F32 residual add (h += X W^T), and the
// fused SwiGLU silu(X Wg^T) * (X Wu^T) (the B tile holds 128 gate rows and
// 128 up rows of the same output columns), stored as BF16 or as a split pair.
//
// Split operands: X may hold each activation as two BF16 halves, x = hi + lo
// with hi = bf16(x) and lo = bf16(x - hi), in columns [0, K) and [K, 2K) of a
// [M, 2K] matrix. The kernel then walks 2K columns of X while the K slabs of W
// wrap around (slab kb of X meets slab kb mod K/64 of W), so one accumulator
// receives hi W^T + lo W^T: the product of the activation to about 2^-17 of
// its value instead of BF16's 2^-9, at twice the tensor work.
#include <cudaTypedefs.h>

#include "kernels.cuh"
#include "sm100.cuh"

namespace clef {

namespace {

using namespace sm100;

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;   // 16 KB
constexpr int B_BYTES = BN * BK * 2;   // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int GROUP_N = 8;
constexpr int EPI_WARPS = 4;
constexpr int THREADS = 64 + EPI_WARPS * 32;
constexpr uint32_t TMEM_COLS = 512;
constexpr size_t SMEM_BYTES = 1024 + (size_t)STAGES * STAGE_BYTES + 256;

struct GemmParams {
  int64_t M;
  int N;        // output columns
  int K;        // columns of X walked by the MMA loop (2 x W's K for split operands)
  int kb_w;     // 64-wide K slabs of W (== K / 64 unless X is split)
  int epi;
  void* out;
  int64_t ldo;
  int tiles_m, tiles_n;
};

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& tm, int& tn) {
  const int per_group = GROUP_N * tiles_m;
  const int group = t / per_group;
  const int first_n = group * GROUP_N;
  const int gn = min(GROUP_N, tiles_n - first_n);
  const int r = t - group * per_group;
  tm = r / gn;
  tn = first_n + r % gn;
}

__device__ __forceinline__ float u2f(uint32_t x) { return __uint_as_float(x); }

// Epilogue of one accumulator row: TMEM row `tbase` (lane quarter and
// accumulator already applied) of output row m, output column tile tn.
__device__ __forceinline__ void store_tile(const GemmParams& p, uint32_t tbase, int64_t m, int tn,
                                           bool swiglu) {
  if (swiglu) {
    uint16_t* out = reinterpret_cast<uint16_t*>(p.out);
#pragma unroll 1
    for (int c = 0; c < 128 / 32; ++c) {
      uint32_t gr[32], ur[32];
      tmem_ld_32x32b_x32(tbase + c * 32, gr);
      tmem_ld_32x32b_x32(tbase + 128 + c * 32, ur);
      tmem_ld_wait();
      const int n0 = tn * 128 + c * 32;
      if (m < p.M) {
        uint32_t packed[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float g0 = u2f(gr[2 * j]), g1 = u2f(gr[2 * j + 1]);
          const float y0 = silu_f(g0) * u2f(ur[2 * j]);
          const float y1 = silu_f(g1) * u2f(ur[2 * j + 1]);
          packed[j] = pack_bf16x2(y0, y1);
        }
        uint16_t* dst = out + m * p.ldo + n0;
        if (n0 + 32 <= p.N) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            reinterpret_cast<uint4*>(dst)[j] =
                make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (n0 + j < p.N) dst[j] = (uint16_t)((packed[j >> 1] >> ((j & 1) * 16)) & 0xffff);
        }
        if (p.epi == kEpiSwiGLUSplit) {
          // Low halves: y - bf16(y), columns [N, 2N) of the row.
          uint32_t low[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float g0 = u2f(gr[2 * j]), g1 = u2f(gr[2 * j + 1]);
            const float y0 = silu_f(g0) * u2f(ur[2 * j]);
            const float y1 = silu_f(g1) * u2f(ur[2 * j + 1]);
            low[j] = pack_bf16x2(y0 - __uint_as_float(packed[j] << 16),
                                 y1 - __uint_as_float(packed[j] & 0xffff0000u));
          }
          uint16_t* dlo = dst + p.N;
          if (n0 + 32 <= p.N) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              reinterpret_cast<uint4*>(dlo)[j] = make_uint4(low[4 * j], low[4 * j + 1], low[4 * j + 2], low[4 * j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (n0 + j < p.N) dlo[j] = (uint16_t)((low[j >> 1] >> ((j & 1) * 16)) & 0xffff);
          }
        }
      }
    }
  } else {
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      const int n0 = tn * BN + c * 32;
      if (n0 >= p.N) break;  // warp-uniform
      uint32_t r[32];
      tmem_ld_32x32b_x32(tbase + c * 32, r);
      tmem_ld_wait();
      if (m >= p.M) continue;
      const bool full_chunk = n0 + 32 <= p.N;
      if (p.epi == kEpiBF16) {
        uint16_t* dst = reinterpret_cast<uint16_t*>(p.out) + m * p.ldo + n0;
        if (full_chunk) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            reinterpret_cast<uint4*>(dst)[j] = make_uint4(
                pack_bf16x2(u2f(r[8 * j]), u2f(r[8 * j + 1])),
                pack_bf16x2(u2f(r[8 * j + 2]), u2f(r[8 * j + 3])),
                pack_bf16x2(u2f(r[8 * j + 4]), u2f(r[8 * j + 5])),
                pack_bf16x2(u2f(r[8 * j + 6]), u2f(r[8 * j + 7])));
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (n0 + j < p.N) dst[j] = f2bf(u2f(r[j]));
        }
      } else {
        float* dst = reinterpret_cast<float*>(p.out) + m * p.ldo + n0;
        if (full_chunk) {
          if (p.epi == kEpiAddF32) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float4 o = reinterpret_cast<float4*>(dst)[j];
              o.x += u2f(r[4 * j]);
              o.y += u2f(r[4 * j + 1]);
              o.z += u2f(r[4 * j + 2]);
              o.w += u2f(r[4 * j + 3]);
              reinterpret_cast<float4*>(dst)[j] = o;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j)
              reinterpret_cast<float4*>(dst)[j] = make_float4(
                  u2f(r[4 * j]), u2f(r[4 * j + 1]), u2f(r[4 * j + 2]), u2f(r[4 * j + 3]));
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (n0 + j < p.N) dst[j] = p.epi == kEpiAddF32 ? dst[j] + u2f(r[j]) : u2f(r[j]);
        }
      }
    }
  }
}

__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const __grid_constant__ CUtensorMap map_b2, GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool swiglu = p.epi == kEpiSwiGLU || p.epi == kEpiSwiGLUSplit;
  const int num_tiles = p.tiles_m * p.tiles_n;
  const int nk = p.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], EPI_WARPS);
    }
    fence_barrier_init();
    tma_prefetch(&map_a);
    tma_prefetch(&map_b);
    if (swiglu) tma_prefetch(&map_b2);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int tm, tn;
        tile_coords(t, p.tiles_m, p.tiles_n, tm, tn);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + (size_t)stage * STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          mbar_expect_tx(&full[stage], STAGE_BYTES);
          const int kw = (kb % p.kb_w) * BK;  // W's slab (wraps for split X)
          tma_load_2d(&map_a, &full[stage], sa, kb * BK, tm * BM);
          if (swiglu) {
            tma_load_2d(&map_b, &full[stage], sb, kw, tn * 128);
            tma_load_2d(&map_b2, &full[stage], sb + B_BYTES / 2, kw, tn * 128);
          } else {
            tma_load_2d(&map_b, &full[stage], sb, kw, tn * BN);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) raise_device_error(kDevGemmTimeout);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full[stage], phase)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + (size_t)stage * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            umma_f16(d, desc_k_sw128(sa + k * 32), desc_k_sw128(sb + k * 32), idesc,
                     (kb | k) != 0);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        umma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (!ok) raise_device_error(kDevGemmTimeout);
    }
  } else {
    // Epilogue warps: TMEM lane quarter is fixed by warp index % 4.
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      int tm, tn;
      tile_coords(t, p.tiles_m, p.tiles_n, tm, tn);
      if (!mbar_wait(&tfull[acc], acc_phase)) {
        raise_device_error(kDevGemmTimeout);
        break;
      }
      tc_fence_after();
      const int64_t m = (int64_t)tm * BM + row_in_tile;
      const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);
      store_tile(p, tbase, m, tn, swiglu);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---- CTA-pair variant ---------------------------------------------------------
// A cluster of two CTAs on neighbouring SMs computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2: CTA r holds A rows [128 r, 128 r + 128) and B rows
// [128 r, 128 r + 128) of the tile (for SwiGLU: CTA 0 the gate rows, CTA 1 the
// up rows), the even CTA issues the MMAs, and each CTA's TMEM receives its own
// 128 rows x 256 columns. Every CTA streams 32 KB per 64-wide K slab instead of
// 48 KB for the same tensor work, so L2 and shared-memory traffic per FLOP drop
// by a third. Both CTAs load their halves with plain (non-multicast) TMA whose
// byte counts land on the even CTA's stage barrier; the MMA completion is
// signalled to both CTAs' barriers by one multicast commit.
constexpr int P_STAGES = 6;
constexpr int P_A_BYTES = 128 * BK * 2;  // 16 KB
constexpr int P_B_BYTES = 128 * BK * 2;  // 16 KB
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;
constexpr size_t P_SMEM_BYTES = 1024 + (size_t)P_STAGES * P_STAGE_BYTES + 256;

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                     const __grid_constant__ CUtensorMap map_b2, GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)P_STAGES * P_STAGE_BYTES);
  uint64_t* empty = full + P_STAGES;
  uint64_t* tfull = empty + P_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  const bool swiglu = p.epi == kEpiSwiGLU || p.epi == kEpiSwiGLUSplit;
  const int num_tiles = p.tiles_m * p.tiles_n;
  const int nk = p.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * EPI_WARPS);  // the epilogue warps of both CTAs
    }
    mbar_init(drain, 1);
    fence_barrier_init();
    tma_prefetch(&map_a);
    tma_prefetch(&map_b);
    if (swiglu) tma_prefetch(&map_b2);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any remote arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t full0 = mapa_shared(&full[0], 0);  // the even CTA's stage barriers
      int stage = 0;
      uint32_t phase = 0;
      for (int t = cluster; t < num_tiles && ok; t += nclusters) {
        int tm, tn;
        tile_coords(t, p.tiles_m, p.tiles_n, tm, tn);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + (size_t)stage * P_STAGE_BYTES;
          uint8_t* sb = sa + P_A_BYTES;
          if (leader) mbar_expect_tx(&full[stage], 2 * P_STAGE_BYTES);
          const uint32_t bar = full0 + (uint32_t)(stage * sizeof(uint64_t));
          const int kw = (kb % p.kb_w) * BK;  // W's slab (wraps for split X)
          tma_load_2d_pair(&map_a, bar, sa, kb * BK, tm * 256 + (int)rank * 128);
          if (swiglu)
            tma_load_2d_pair(leader ? &map_b : &map_b2, bar, sb, kw, tn * 128);
          else
            tma_load_2d_pair(&map_b, bar, sb, kw, tn * BN + (int)rank * 128);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) raise_device_error(kDevGemmTimeout);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = idesc_bf16_f32(256, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool issued = false;
      for (int t = cluster; t < num_tiles && ok; t += nclusters) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full[stage], phase)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + (size_t)stage * P_STAGE_BYTES);
          const uint32_t sb = sa + P_A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16_pair(d, desc_k_sw128(sa + k * 32), desc_k_sw128(sb + k * 32), idesc, (kb | k) != 0);
          issued = true;
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[acc], 0x3);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (!ok) {
        // The MMAs already issued write both CTAs' TMEM: let them finish
        // (bounded) before the allocation is released.
        raise_device_error(kDevGemmTimeout);
        if (issued) {
          umma_commit_pair(drain, 0x1);
          mbar_wait(drain, 0);
        }
      }
    }
  } else {
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t tempty0 = mapa_shared(&tempty[0], 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = cluster; t < num_tiles; t += nclusters) {
      int tm, tn;
      tile_coords(t, p.tiles_m, p.tiles_n, tm, tn);
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase))) {
        raise_device_error(kDevGemmTimeout);
        break;
      }
      tc_fence_after();
      const int64_t m = (int64_t)tm * 256 + rank * 128 + row_in_tile;
      const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);
      store_tile(p, tbase, m, tn, swiglu);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty0 + (uint32_t)(acc * sizeof(uint64_t)));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA releases TMEM or exits while its pair still uses it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// Row-major BF16 [rows, cols] matrix, box = box_rows x 64 columns, 128-byte swizzle.
int make_map(CUtensorMap* map, const void* ptr, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail(CLEF_ERR_CUDA, "gemm: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(CLEF_ERR_CUDA, "gemm: cuTensorMapEncodeTiled failed");
  return CLEF_OK;
}

}  // namespace

int launch_gemm(const uint16_t* X, const uint16_t* W, const uint16_t* W2, int64_t M, int N, int K,
                int epi, void* out, int64_t ldo, cudaStream_t s, int x_split) {
  if (M == 0) return CLEF_OK;
  CLEF_CHECK(K % BK == 0 && K > 0, CLEF_ERR_UNSUPPORTED, "gemm: K must be a multiple of 64");
  CLEF_CHECK(N > 0 && N % 16 == 0, CLEF_ERR_UNSUPPORTED, "gemm: N must be a multiple of 16");
  CLEF_CHECK(M <= (int64_t)INT32_MAX - BM, CLEF_ERR_UNSUPPORTED, "gemm: M too large");
  CLEF_CHECK(((uintptr_t)X & 15) == 0 && ((uintptr_t)W & 15) == 0 && ((uintptr_t)out & 15) == 0,
             CLEF_ERR_INVALID, "gemm: operands must be 16-byte aligned");
  const bool swiglu = epi == kEpiSwiGLU || epi == kEpiSwiGLUSplit;
  const int elem = (epi == kEpiBF16 || swiglu) ? 2 : 4;
  const int out_cols = epi == kEpiSwiGLUSplit ? 2 * N : N;
  CLEF_CHECK(ldo >= out_cols && (ldo * elem) % 16 == 0, CLEF_ERR_INVALID,
             "gemm: ldo must cover the output columns and keep rows 16-byte aligned");
  CUtensorMap ma, mb, mb2;
  const bool pair_maps = M > BM;  // the CTA-pair kernel loads 128-row halves of B
  const int xk = x_split ? 2 * K : K;  // columns of X (hi | lo halves when split)
  int rc = make_map(&ma, X, (uint64_t)M, (uint64_t)xk, BM);
  if (rc) return rc;
  if (swiglu) {
    CLEF_CHECK(W2 && ((uintptr_t)W2 & 15) == 0, CLEF_ERR_INVALID, "gemm: SwiGLU up matrix");
    rc = make_map(&mb, W, (uint64_t)N, (uint64_t)K, 128);
    if (!rc) rc = make_map(&mb2, W2, (uint64_t)N, (uint64_t)K, 128);
  } else {
    rc = make_map(&mb, W, (uint64_t)N, (uint64_t)K, pair_maps ? 128 : BN);
    mb2 = mb;
  }
  if (rc) return rc;
  const bool pair = M > BM;
  GemmParams p;
  p.M = M;
  p.N = N;
  p.K = xk;
  p.kb_w = K / BK;
  p.epi = epi;
  p.out = out;
  p.ldo = ldo;
  p.tiles_m = (int)ceil_div(M, pair ? 256 : BM);
  p.tiles_n = (int)ceil_div(N, swiglu ? 128 : BN);
  int dev = 0;
  CLEF_CUDA(cudaGetDevice(&dev));
  static bool attr[64] = {false};
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    CLEF_CUDA(cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)SMEM_BYTES));
    CLEF_CUDA(cudaFuncSetAttribute(gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)P_SMEM_BYTES));
    attr[dev] = true;
  }
  const int tiles = p.tiles_m * p.tiles_n;
  if (pair) {
    const int clusters = std::min(tiles, std::max(1, persistent_ctas(dev) / 2));
    gemm_pair_kernel<<<2 * clusters, THREADS, P_SMEM_BYTES, s>>>(ma, mb, mb2, p);
    return launch_status("gemm_pair");
  }
  const int grid = std::min(tiles, persistent_ctas(dev));
  gemm_kernel<<<grid, THREADS, SMEM_BYTES, s>>>(ma, mb, mb2, p);
  return launch_status("gemm");
}

int gemm_device_error(int* code) { return read_device_error(code); }

}  // namespace clef

using namespace clef;

extern "C" {

int clef_gemm_bf16(const uint16_t* X, const uint16_t* W, int64_t M, int32_t N, int32_t K,
                   int32_t epilogue, void* out, int64_t ldo, void* stream) {
  CLEF_CHECK(X && W && out, CLEF_ERR_INVALID, "gemm_bf16: null pointer");
  CLEF_CHECK(M >= 0, CLEF_ERR_INVALID, "gemm_bf16: M");
  CLEF_CHECK(epilogue >= CLEF_EPI_STORE_BF16 && epilogue <= CLEF_EPI_ADD_F32, CLEF_ERR_INVALID,
             "gemm_bf16: epilogue");
  return launch_gemm(X, W, nullptr, M, N, K, epilogue, out, ldo, as_stream(stream));
}

int clef_gemm_bf16_split(const uint16_t* X2, const uint16_t* W, int64_t M, int32_t N, int32_t K,
                         int32_t epilogue, void* out, int64_t ldo, void* stream) {
  CLEF_CHECK(X2 && W && out, CLEF_ERR_INVALID, "gemm_bf16_split: null pointer");
  CLEF_CHECK(M >= 0, CLEF_ERR_INVALID, "gemm_bf16_split: M");
  CLEF_CHECK(epilogue >= CLEF_EPI_STORE_BF16 && epilogue <= CLEF_EPI_ADD_F32, CLEF_ERR_INVALID,
             "gemm_bf16_split: epilogue");
  return launch_gemm(X2, W, nullptr, M, N, K, epilogue, out, ldo, as_stream(stream), 1);
}

int clef_gemm_swiglu(const uint16_t* X, const uint16_t* Wg, const uint16_t* Wu, int64_t M,
                     int32_t N, int32_t K, uint16_t* out, void* stream) {
  CLEF_CHECK(X && Wg && Wu && out, CLEF_ERR_INVALID, "gemm_swiglu: null pointer");
  CLEF_CHECK(M >= 0, CLEF_ERR_INVALID, "gemm_swiglu: M");
  return launch_gemm(X, Wg, Wu, M, N, K, kEpiSwiGLU, out, N, as_stream(stream));
}

}  // extern "C"
