// copy_rate.cu — measures what the dual GEMM's producers depend on: the
// cycles a thread spends issuing one bulk global->shared copy, and the
// global->shared bandwidth an SM gets while a given number of SMs copy at
// once (maintainer tool, built and run by nvfp4_dual_gemm_b200.copyrate).
//
// Each CTA (one per SM: 64 KiB of dynamic shared memory, 1 block/SM)
// copies 512 KiB out of its own 64 KiB window of a global buffer into a
// 64 KiB shared ring with `cp.async.bulk`, from `issuers` warps (lane 0
// each), all copies counted on one mbarrier; the wait is bounded.  Every
// address stays inside the CTA's window and ring: copy i reads and writes
// offset (i * bytes) % 64 KiB, bytes a power of two <= 16 KiB.
#include <cstdint>
#include <cstdio>
#include <cstdlib>

#include <cuda_runtime.h>

namespace {

constexpr int kWindow = 65536;
constexpr uint32_t kTotal = 1u << 19;  // bytes per CTA (< 2^20 tx limit)
constexpr long long kWaitLimit = 2000000000ll;

__device__ __forceinline__ uint32_t saddr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ long long cycles() {
  long long t;
  asm volatile("mov.u64 %0, %%clock64;" : "=l"(t));
  return t;
}

__global__ void __launch_bounds__(128, 1)
    copy_rate_kernel(const uint8_t* g, int bytes, int issuers,
                     long long* out) {
  extern __shared__ __align__(1024) uint8_t ring[];
  __shared__ __align__(8) uint64_t bar;
  const int tid = threadIdx.x;
  const int copies = static_cast<int>(kTotal / bytes);
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&bar)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
            saddr(&bar)),
        "r"(kTotal)
        : "memory");
  }
  __syncthreads();
  const uint8_t* src = g + static_cast<size_t>(blockIdx.x) * kWindow;
  const long long t0 = cycles();
  long long t1 = t0;
  if (tid % 32 == 0 && tid / 32 < issuers) {
    for (int i = tid / 32; i < copies; i += issuers) {
      const uint32_t off = static_cast<uint32_t>((i * bytes) % kWindow);
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
          "[%0], [%1], %2, [%3];" ::"r"(saddr(ring + off)),
          "l"(src + off), "r"(bytes), "r"(saddr(&bar))
          : "memory");
    }
    t1 = cycles();
  }
  uint32_t done = 0;
  while (!done && cycles() - t0 < kWaitLimit) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(saddr(&bar))
        : "memory");
  }
  const long long t2 = cycles();
  if (tid == 0) {
    out[3 * blockIdx.x + 0] = t1 - t0;  // issue time of warp 0's copies
    out[3 * blockIdx.x + 1] = t2 - t0;  // time until all bytes landed
    out[3 * blockIdx.x + 2] = done;
  }
}

// Distributed-shared-memory exchange rate (the cluster split-K epilogue's
// pattern): clusters of two CTAs, each sending the 64 KiB at the start of
// its shared memory into the second 64 KiB of its peer's, either as bulk
// copies (mode 0: lane 0 of `issuers` warps, `bytes` per copy) or as
// 16-byte st.async stores from all 256 threads (mode 1).  Both directions
// run at once; the bytes count on the receiver's mbarrier, whose bounded
// wait ends the timing.  Every address stays inside the 128 KiB buffer.
constexpr uint32_t kX = 65536;

__global__ void __launch_bounds__(256, 1)
    dsmem_rate_kernel(int mode, int bytes, int issuers, long long* out) {
  extern __shared__ __align__(1024) uint8_t buf[];  // [out 64K][in 64K]
  __shared__ __align__(8) uint64_t bar;
  const int tid = threadIdx.x;
  uint32_t rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  const uint32_t peer = rank ^ 1u;
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&bar)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
            saddr(&bar)),
        "r"(kX)
        : "memory");
  }
  __syncthreads();
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
  uint32_t dst, pbar;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
               : "=r"(dst) : "r"(saddr(buf + kX)), "r"(peer));
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
               : "=r"(pbar) : "r"(saddr(&bar)), "r"(peer));
  const long long t0 = cycles();
  if (mode == 0) {
    if (tid % 32 == 0 && tid / 32 < issuers) {
      const int copies = static_cast<int>(kX / bytes);
      for (int i = tid / 32; i < copies; i += issuers)
        asm volatile(
            "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::"
            "bytes [%0], [%1], %2, [%3];" ::"r"(dst + i * bytes),
            "r"(saddr(buf) + i * bytes), "r"(bytes), "r"(pbar)
            : "memory");
    }
  } else {
    for (int j = 0; j < static_cast<int>(kX / 16 / 256); ++j) {
      const uint32_t off = static_cast<uint32_t>((j * 256 + tid) * 16);
      asm volatile(
          "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 "
          "[%0], {%1, %2, %3, %4}, [%5];" ::"r"(dst + off),
          "r"(off), "r"(off + 1), "r"(off + 2), "r"(off + 3), "r"(pbar)
          : "memory");
    }
  }
  uint32_t done = 0;
  while (!done && cycles() - t0 < kWaitLimit) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(saddr(&bar))
        : "memory");
  }
  const long long t1 = cycles();
  // no CTA leaves while its peer may still write into it
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
  if (tid == 0) {
    out[2 * blockIdx.x + 0] = t1 - t0;
    out[2 * blockIdx.x + 1] = done;
  }
}

int check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    std::fprintf(stderr, "%s: %s\n", what, cudaGetErrorString(e));
    return 1;
  }
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  int sms = 0;
  if (check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0),
            "cudaDeviceGetAttribute"))
    return 1;
  uint8_t* g = nullptr;
  long long* d_out = nullptr;
  if (check(cudaMalloc(&g, static_cast<size_t>(sms) * kWindow), "cudaMalloc") ||
      check(cudaMemset(g, 1, static_cast<size_t>(sms) * kWindow), "cudaMemset") ||
      check(cudaMalloc(&d_out, sizeof(long long) * 3 * sms), "cudaMalloc") ||
      check(cudaFuncSetAttribute(copy_rate_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kWindow),
            "cudaFuncSetAttribute"))
    return 1;
  long long* h = static_cast<long long*>(std::malloc(sizeof(long long) * 3 * sms));
  const int ctas_list[] = {1, 32, 64, 96, 128, sms};
  const int bytes_list[] = {2048, 16384};
  const int issuers_list[] = {1, 2, 4};
  std::printf("ctas,bytes,issuers,issue_cycles_per_copy,cycles_per_copy,"
              "bytes_per_cycle_per_sm,ok\n");
  for (int ctas : ctas_list) {
    for (int bytes : bytes_list) {
      for (int issuers : issuers_list) {
        for (int rep = 0; rep < 2; ++rep) {  // first run warms L2
          copy_rate_kernel<<<ctas, 128, kWindow>>>(g, bytes, issuers, d_out);
          if (check(cudaDeviceSynchronize(), "copy_rate_kernel")) return 1;
        }
        if (check(cudaMemcpy(h, d_out, sizeof(long long) * 3 * ctas,
                             cudaMemcpyDeviceToHost),
                  "cudaMemcpy"))
          return 1;
        double issue = 0, total = 0;
        long long ok = 1;
        for (int c = 0; c < ctas; ++c) {
          issue += static_cast<double>(h[3 * c]);
          total += static_cast<double>(h[3 * c + 1]);
          ok &= h[3 * c + 2];
        }
        const int copies = static_cast<int>(kTotal / bytes);
        issue /= ctas;
        total /= ctas;
        std::printf("%d,%d,%d,%.1f,%.1f,%.1f,%lld\n", ctas, bytes, issuers,
                    issue / ((copies + issuers - 1) / issuers),
                    total / copies, kTotal / total, ok);
      }
    }
  }
  // DSMEM exchange: 64 clusters of two (128 CTAs, as the C2 split-K plan)
  if (check(cudaFuncSetAttribute(dsmem_rate_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 2 * kX),
            "cudaFuncSetAttribute"))
    return 1;
  std::printf("dsmem_mode,bytes,issuers,cycles_for_64KiB,bytes_per_cycle_per_sm,ok\n");
  const int modes[][3] = {{0, 4096, 8}, {0, 16384, 4}, {0, 8192, 8},
                          {0, 65536, 1}, {1, 16, 256}};
  for (const auto& m : modes) {
    const int ctas = 128;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas, 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.dynamicSmemBytes = 2 * kX;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    for (int rep = 0; rep < 2; ++rep) {
      if (check(cudaLaunchKernelEx(&cfg, dsmem_rate_kernel, m[0], m[1], m[2],
                                   d_out),
                "dsmem_rate_kernel") ||
          check(cudaDeviceSynchronize(), "dsmem_rate_kernel"))
        return 1;
    }
    if (check(cudaMemcpy(h, d_out, sizeof(long long) * 2 * ctas,
                         cudaMemcpyDeviceToHost),
              "cudaMemcpy"))
      return 1;
    double total = 0;
    long long ok = 1;
    for (int c = 0; c < ctas; ++c) {
      total += static_cast<double>(h[2 * c]);
      ok &= h[2 * c + 1];
    }
    total /= ctas;
    std::printf("%s,%d,%d,%.0f,%.1f,%lld\n", m[0] ? "st.async" : "bulk",
                m[1], m[2], total, kX / total, ok);
  }
  std::free(h);
  cudaFree(d_out);
  cudaFree(g);
  return 0;
}
