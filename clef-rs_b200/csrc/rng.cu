// rng.cu — seeded synthetic parameters. Philox4x32-10 (Salmon, Moraes, Dror,
// Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC 2011) maps
// (counter, key) to four 32-bit words; the Box-Muller transform turns two
// uniforms into two standard normals. Element i of a tensor uses counter
// (i / 4, stream) and key = seed, so values do not depend on the launch shape
// or on the host thread count.
#include <cmath>
#include <thread>
#include <vector>

#include "kernels.cuh"

namespace clef {

namespace {

struct U4 {
  uint32_t x, y, z, w;
};

__host__ __device__ inline void mulhilo(uint32_t a, uint32_t b, uint32_t& hi, uint32_t& lo) {
  const uint64_t p = (uint64_t)a * (uint64_t)b;
  hi = (uint32_t)(p >> 32);
  lo = (uint32_t)p;
}

__host__ __device__ inline U4 philox(U4 c, uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
  for (int r = 0; r < 10; ++r) {
    uint32_t hi0, lo0, hi1, lo1;
    mulhilo(M0, c.x, hi0, lo0);
    mulhilo(M1, c.z, hi1, lo1);
    c = U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
    k0 += W0;
    k1 += W1;
  }
  return c;
}

// Uniform in (0, 1]: (u + 1) * 2^-32 never reaches 0, so log() is finite.
__host__ __device__ inline float unit(uint32_t u) { return ((float)u + 1.0f) * 2.3283064365386963e-10f; }

__host__ __device__ inline void normals(uint64_t seed, uint64_t stream, uint64_t block, float out[4]) {
  const U4 c{(uint32_t)block, (uint32_t)(block >> 32), (uint32_t)stream, (uint32_t)(stream >> 32)};
  const U4 r = philox(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  const float u0 = unit(r.x), u1 = unit(r.y), u2 = unit(r.z), u3 = unit(r.w);
  const float a = sqrtf(-2.0f * logf(u0)), b = sqrtf(-2.0f * logf(u2));
  const float t1 = 6.283185307179586f * u1, t3 = 6.283185307179586f * u3;
  out[0] = a * cosf(t1);
  out[1] = a * sinf(t1);
  out[2] = b * cosf(t3);
  out[3] = b * sinf(t3);
}

__host__ __device__ inline void uniforms(uint64_t seed, uint64_t stream, uint64_t block, float out[4]) {
  const U4 c{(uint32_t)block, (uint32_t)(block >> 32), (uint32_t)stream, (uint32_t)(stream >> 32)};
  const U4 r = philox(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  out[0] = unit(r.x);
  out[1] = unit(r.y);
  out[2] = unit(r.z);
  out[3] = unit(r.w);
}

__global__ void fill_normal_bf16_kernel(uint16_t* __restrict__ dst, int64_t n, uint64_t seed,
                                        uint64_t stream, float mean, float std) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b * 4 < n; b += stride) {
    float z[4];
    normals(seed, stream, (uint64_t)b, z);
    for (int j = 0; j < 4; ++j) {
      const int64_t i = b * 4 + j;
      if (i < n) dst[i] = f2bf(mean + std * z[j]);
    }
  }
}

}  // namespace

uint64_t name_stream(const char* name) {  // FNV-1a 64
  uint64_t h = 1469598103934665603ull;
  for (const char* p = name; *p; ++p) {
    h ^= (uint8_t)*p;
    h *= 1099511628211ull;
  }
  return h;
}

int launch_fill_normal_bf16(uint16_t* dst, int64_t n, uint64_t seed, uint64_t stream, float mean,
                            float std, cudaStream_t s) {
  if (n == 0) return CLEF_OK;
  const int64_t blocks4 = ceil_div(n, 4);
  const unsigned grid = (unsigned)std::min<int64_t>(ceil_div(blocks4, 256), 148 * 16);
  fill_normal_bf16_kernel<<<grid, 256, 0, s>>>(dst, n, seed, stream, mean, std);
  return launch_status("fill_normal_bf16");
}

void host_fill(float* dst, int64_t n, uint64_t seed, uint64_t stream, int kind, float a, float b) {
  const int64_t blocks = ceil_div(n, 4);
  auto work = [&](int64_t b0, int64_t b1) {
    for (int64_t blk = b0; blk < b1; ++blk) {
      float z[4];
      if (kind == kFillNormal) normals(seed, stream, (uint64_t)blk, z);
      else uniforms(seed, stream, (uint64_t)blk, z);
      for (int j = 0; j < 4; ++j) {
        const int64_t i = blk * 4 + j;
        if (i < n) dst[i] = kind == kFillNormal ? a + b * z[j] : a + (b - a) * z[j];
      }
    }
  };
  const int64_t threads = blocks > (1 << 16) ? 8 : 1;
  if (threads == 1) {
    work(0, blocks);
    return;
  }
  std::vector<std::thread> pool;
  for (int64_t t = 0; t < threads; ++t)
    pool.emplace_back(work, blocks * t / threads, blocks * (t + 1) / threads);
  for (auto& th : pool) th.join();
}

}  // namespace clef
