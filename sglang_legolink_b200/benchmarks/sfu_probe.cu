// Per-SM throughput of the softmax building blocks on this GPU: exp2 on the
// MUFU pipe, the polynomial exp2 of the attention kernel (FMA / ALU pipes),
// the bf16x2 pack, FFMA, and MUFU / polynomial mixes.  One block per SM, 16
// independent chains per thread; element-ops per clock per SM from clock64.
// Built and run by sfu_probe.py.
#include <cstdio>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

__device__ __forceinline__ float ex2(float x) { float y; asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x)); return y; }
__device__ __forceinline__ float exp2_poly(float x) {
  x = fmaxf(x, -126.f);
  const float t = __fadd_rn(x, 12582912.f);
  const float f = __fsub_rn(x, __fsub_rn(t, 12582912.f));
  float p = fmaf(f, 0.05517166f, 0.24261113f);
  p = fmaf(p, f, 0.69326097f);
  p = fmaf(p, f, 0.99992806f);
  return __uint_as_float(__float_as_uint(p) + (__float_as_uint(t) << 23));
}
__device__ __forceinline__ uint32_t pack(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

constexpr int CH = 16;   // independent chains per thread
constexpr int IT = 512;  // iterations

template <int MODE>
__global__ void probe(float* out, unsigned long long* cyc, float seed) {
  float v[CH];
#pragma unroll
  for (int i = 0; i < CH; ++i) v[i] = seed * (threadIdx.x + i) * 1e-6f - 1.f;
  uint32_t acc = 0;
  __syncthreads();
  unsigned long long t0 = clock64();
  for (int it = 0; it < IT; ++it) {
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      if (MODE == 0) v[i] = ex2(v[i]) - 1.5f;                         // MUFU (+1 FADD)
      if (MODE == 1) v[i] = exp2_poly(v[i]) - 1.5f;                   // poly
      if (MODE == 2) v[i] = fmaf(v[i], 0.999f, -0.001f);              // FFMA only
      if (MODE == 3) { acc += pack(v[i], v[i] * 0.5f); v[i] = v[i] * 0.9999f; }  // F2FP + FMUL
      if (MODE == 4) v[i] = ((i & 3) == 0 ? exp2_poly(v[i]) : ex2(v[i])) - 1.5f;  // 25 % poly
      if (MODE == 5) v[i] = ((i & 1) == 0 ? exp2_poly(v[i]) : ex2(v[i])) - 1.5f;  // 50 % poly
      if (MODE == 6) { float e = ex2(v[i]); acc += pack(e, e); v[i] = e - 1.5f; }  // ex2 + pack
    }
  }
  __syncthreads();
  unsigned long long t1 = clock64();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < CH; ++i) s += v[i];
  out[blockIdx.x * blockDim.x + threadIdx.x] = s + (float)acc;
  if (threadIdx.x == 0) cyc[blockIdx.x] = t1 - t0;
}

template <int MODE>
void run(const char* name, int threads) {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  const int blocks = sms;  // one block per SM
  float* out; unsigned long long* cyc;
  cudaMalloc(&out, blocks * threads * sizeof(float));
  cudaMalloc(&cyc, blocks * sizeof(unsigned long long));
  probe<MODE><<<blocks, threads>>>(out, cyc, 1.f);
  probe<MODE><<<blocks, threads>>>(out, cyc, 1.f);
  cudaDeviceSynchronize();
  unsigned long long h[1024];
  cudaMemcpy(h, cyc, blocks * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
  double mean = 0; for (int i = 0; i < blocks; ++i) mean += h[i]; mean /= blocks;
  const double ops = (double)threads * CH * IT;
  printf("{\"mode\": \"%s\", \"threads\": %d, \"cycles\": %.0f, \"elem_ops_per_clk_per_sm\": %.2f}\n", name, threads,
         mean, ops / mean);
  cudaFree(out); cudaFree(cyc);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) printf("error %s\n", cudaGetErrorString(e));
}

int main() {
  for (int th : {256, 512, 1024}) {
    run<0>("ex2", th);
    run<1>("poly", th);
    run<2>("ffma", th);
    run<3>("pack_bf16x2+fmul", th);
    run<4>("ex2_75_poly_25", th);
    run<5>("ex2_50_poly_50", th);
    run<6>("ex2+pack", th);
  }
  return 0;
}
