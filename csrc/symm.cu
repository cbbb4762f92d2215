// Symmetric peer memory over NVLink / NVSwitch and the collective kernels that use it (sm_100a).
//
// Every rank cudaMallocs one buffer of the same size, exports a CUDA IPC handle, and maps the
// peers' buffers (exchanged over torch.distributed) with cudaIpcOpenMemHandle, so a kernel can
// load from and store to any peer's memory with ordinary P2P instructions.  A small flag array
// per rank carries monotonically increasing epochs: rank r signals an epoch to every peer by
// storing it into flag[r] of the peer's array (release, system scope) and waits until its own
// array shows at least that epoch from every peer (acquire, bounded: after the poll budget the
// kernel records an error code in `err` and carries on instead of hanging).
//
//   allreduce   one-shot all-reduce of a bf16 vector already in each rank's symmetric buffer:
//               barrier, then every rank reads all peers' copies over NVLink, sums in fp32, adds an
//               optional residual and writes its own output.  Callers alternate between two
//               buffers, so one barrier per call suffices (a rank only overwrites a buffer after
//               every peer has entered the next all-reduce, i.e. finished reading it).
//   rs_sumsq    reduce-scatter of fp32 gradient buffers: every rank reads its shard of all peers'
//               gradients, sums, scales, stores (or adds) the shard and its sum of squares;
//               optionally a closing barrier so the source buffer can be reused right after.
//   adamw_ag    sharded AdamW on the reduced shard with the bf16 result stored straight into
//               every peer's parameter buffer (the all-gather fused into the update), then a
//               closing barrier so no rank reads parameters that are still being written.
//   rs_norm_ag  tensor-parallel sequence-parallel boundary: reduce-scatter of a row-parallel
//               GEMM's partials, residual add and RMSNorm on the owned rows, all-gather of the
//               normalised rows by P2P stores, between two barriers.
// No collective here uses TMA or multicast; NCCL stays the baseline path.
#include <cuda_runtime.h>

#include "common.cuh"
#include "ops.h"

namespace trida {
namespace symm {

constexpr int MAXR = 8;
constexpr long long kMaxPolls = 20000000;     // ~ a few seconds with the back-off below

struct Peers {
  void* buf[MAXR];        // symmetric data buffers (this rank's at index rank)
  unsigned* flag[MAXR];   // flag arrays: flag[p][src] = latest epoch signalled by src to p
};

__device__ __forceinline__ void st_release(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Signal `epoch` to every peer (one thread), then every CTA waits for all peers' signals.
__device__ void barrier(const Peers& P, int rank, int world, unsigned epoch, int slot, int* err, int code) {
  if (blockIdx.x == 0 && threadIdx.x < world) {
    __threadfence_system();
    st_release(P.flag[threadIdx.x] + slot * MAXR + rank, epoch);
  }
  if (threadIdx.x < world) {
    const unsigned* f = P.flag[rank] + slot * MAXR + threadIdx.x;
    long long polls = 0;
    while ((int)(ld_acquire(f) - epoch) < 0) {
      if (++polls > kMaxPolls) {
        atomicExch(err, code);
        break;
      }
      if (polls > 64) __nanosleep(256);
    }
  }
  __syncthreads();
}

// `ctr` (this rank's device counter) supplies the epoch, so a call captured in a CUDA graph takes
// a fresh epoch on every replay; the last CTA to finish advances the counter.
__global__ void allreduce_kernel(Peers P, int rank, int world, unsigned* ctr, unsigned* done, int64_t off, int64_t n,
                                 const bf16* residual, bf16* out, int* err) {
  const unsigned epoch = *reinterpret_cast<volatile unsigned*>(ctr) + 1;
  barrier(P, rank, world, epoch, 0, err, 201);
  const int64_t n8 = n / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < world; ++r) {
      const int src = (rank + r) % world;     // stagger the peers each rank reads first
      float v[8];
      load8(reinterpret_cast<const bf16*>(P.buf[src]) + off + i * 8, v);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += v[e];
    }
    if (residual != nullptr) {
      float rv[8];
      load8(residual + i * 8, rv);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += rv[e];
    }
    store8(out + i * 8, acc);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *done = 0;
      *ctr = epoch;
      __threadfence();
    }
  }
}

// close_slot >= 0: a closing barrier on that flag slot -- the last CTA to finish reading signals
// every peer and waits for theirs, so when the kernel completes no rank still reads this rank's
// gradient buffer (it may be reused at once).
__global__ void rs_sumsq_kernel(Peers P, int rank, int world, unsigned epoch, int64_t shard_off, int64_t shard_len,
                                float scale, float* shard_out, float* partial, int accumulate, int* err,
                                unsigned* done, int close_slot) {
  barrier(P, rank, world, epoch, 1, err, 202);
  float ss = 0.f;
  const int64_t n4 = shard_len / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < world; ++r) {
      const int src = (rank + r) % world;
      const float4 v = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(P.buf[src]) + shard_off)[i];
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    acc.x *= scale; acc.y *= scale; acc.z *= scale; acc.w *= scale;
    if (accumulate) {
      const float4 o = reinterpret_cast<const float4*>(shard_out)[i];
      acc.x += o.x; acc.y += o.y; acc.z += o.z; acc.w += o.w;
    }
    reinterpret_cast<float4*>(shard_out)[i] = acc;
    ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
  }
  __shared__ float sred[32];
  ss = block_sum(ss, sred);
  if (threadIdx.x == 0) partial[blockIdx.x] = ss;
  if (close_slot >= 0 && threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *done = 0u;
      __threadfence_system();
      for (int r = 0; r < world; ++r) st_release(P.flag[r] + close_slot * MAXR + rank, epoch);
      for (int r = 0; r < world; ++r) {
        const unsigned* f = P.flag[rank] + close_slot * MAXR + r;
        long long polls = 0;
        while ((int)(ld_acquire(f) - epoch) < 0) {
          if (++polls > kMaxPolls) {
            atomicExch(err, 206);
            break;
          }
          if (polls > 64) __nanosleep(256);
        }
      }
    }
  }
}

__global__ void adamw_ag_kernel(Peers P, int rank, int world, unsigned epoch, int64_t shard_off, int64_t shard_len,
                                const float* grad, float* master, float* m, float* v, float lr, float b1, float b2,
                                float eps, float wd, float bc1, float bc2, const float* coef, unsigned* done,
                                int* err) {
  const float c = coef != nullptr ? *coef : 1.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < shard_len; i += (int64_t)gridDim.x * blockDim.x) {
    const float g = grad[i] * c;
    const float mi = b1 * m[i] + (1.f - b1) * g;
    const float vi = b2 * v[i] + (1.f - b2) * g * g;
    m[i] = mi;
    v[i] = vi;
    float p = master != nullptr ? master[i]
                                : __bfloat162float(reinterpret_cast<const bf16*>(P.buf[rank])[shard_off + i]);
    p *= 1.f - lr * wd;
    p -= lr * (mi / bc1) / (sqrtf(vi / bc2) + eps);
    if (master != nullptr) master[i] = p;
    const bf16 pb = __float2bfloat16(p);
    for (int r = 0; r < world; ++r) reinterpret_cast<bf16*>(P.buf[r])[shard_off + i] = pb;
  }
  // closing barrier: the last CTA to finish signals the peers, every CTA of the *next* use waits
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(done, 1u);
    if (prev == gridDim.x - 1) {
      *done = 0;
      for (int r = 0; r < world; ++r) st_release(P.flag[r] + 2 * MAXR + rank, epoch);
      const unsigned* f = P.flag[rank] + 2 * MAXR;
      for (int r = 0; r < world; ++r) {
        long long polls = 0;
        while ((int)(ld_acquire(f + r) - epoch) < 0) {
          if (++polls > kMaxPolls) {
            atomicExch(err, 203);
            break;
          }
          if (polls > 64) __nanosleep(256);
        }
      }
    }
  }
}

// Global gradient norm from every rank's per-block partial sums of squares (symmetric scratch
// arrays of `nblocks` floats) and the clip coefficient min(1, max_norm / (norm + 1e-6)).
__global__ void norm_coef_kernel(Peers P, int rank, int world, unsigned epoch, int nblocks, float max_norm,
                                 float* norm_out, float* coef_out, int* err) {
  barrier(P, rank, world, epoch, 3, err, 204);
  float s = 0.f;
  for (int r = 0; r < world; ++r)
    for (int i = threadIdx.x; i < nblocks; i += blockDim.x) s += reinterpret_cast<const float*>(P.buf[r])[i];
  __shared__ float sred[32];
  s = block_sum(s, sred);
  if (threadIdx.x == 0) {
    const float nrm = sqrtf(s);
    *norm_out = nrm;
    *coef_out = fminf(1.f, max_norm / (nrm + 1e-6f));
  }
}

// All-gather of one parameter group for full-shard data parallelism: rank r's bf16 shard lives
// at bufs[r] (shard_len elements); every rank copies all shards, in rank order, into its own
// `dst` with 16-byte P2P loads (plain loads through NVLink; no TMA, no multicast).  Consistency
// comes from the callers: a shard only changes in the optimizer step, which ends with barrier();
// the gathers of the next step run after it on every rank.
// Each thread keeps GU 16-byte peer loads in flight before storing them: a load over NVLink takes
// microseconds, so the link needs megabytes in flight per GPU (32 CTAs x 256 threads x 16 x 16 B = 2 MB),
// where one load per thread (128 KB) reached 46 GB/s.
constexpr int GU = 16;
__global__ void gather_kernel(Peers P, int rank, int world, int64_t shard_len, bf16* __restrict__ dst) {
  const int64_t n8 = shard_len / 8;
  const int64_t total = n8 * world;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t base = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < total; base += stride * GU) {
    uint4 v[GU];
#pragma unroll
    for (int u = 0; u < GU; ++u) {
      const int64_t i = base + u * stride;
      if (i < total) {
        const int64_t k = i / n8, j = i - k * n8;
        const int src = (int)((k + rank) % world);      // stagger the peers each rank reads first
        v[u] = reinterpret_cast<const uint4*>(P.buf[src])[j];
      }
    }
#pragma unroll
    for (int u = 0; u < GU; ++u) {
      const int64_t i = base + u * stride;
      if (i < total) {
        const int64_t k = i / n8, j = i - k * n8;
        const int src = (int)((k + rank) % world);
        reinterpret_cast<uint4*>(dst + (int64_t)src * shard_len)[j] = v[u];
      }
    }
  }
}

// Sequence-parallel boundary after a row-parallel GEMM (tensor-parallel serving).  Every rank holds
// its partial product [M, D] in its symmetric buffer P.buf[rank]; rank r owns rows [row0, row0 +
// nrows) of the residual stream (`xs`, bf16, local).  One kernel does the reduce-scatter, the
// residual add, the next sublayer's RMSNorm and the all-gather of its input:
//   opening barrier (every rank's partial is written), then per owned row: sum the W partial rows
//   (P2P loads, fp32), add the residual row, round to bf16 into `xs`, RMSNorm with `w`, and store
//   the normalised row into every rank's gather buffer H[k] (P2P stores); closing barrier (the last
//   CTA of each rank signals every peer once all its rows are out and waits for theirs), so when
//   the kernel completes this rank's gather buffer holds all M normalised rows and no peer still
//   reads this rank's partial buffer.
// Bytes per rank over NVLink: (W-1)/W of the partial in and (W-1)/W of the normalised rows out --
// half of what a one-shot all-reduce reads at W = 2 and 2/W of it in general.  Each row is reduced
// by exactly one rank, so every rank sees bitwise the same normalised rows.
struct PeerBufs {
  void* p[MAXR];
};

__device__ __forceinline__ uint32_t pk2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
constexpr int SP_OPEN = 6, SP_CLOSE = 7;   // flag slots of the two barriers

__global__ void rs_norm_ag_kernel(Peers P, PeerBufs H, int rank, int world, unsigned* ctr, int D, int64_t row0,
                                  int nrows, bf16* __restrict__ xs, const bf16* __restrict__ w, float eps, int* err) {
  const unsigned epoch = *reinterpret_cast<volatile unsigned*>(ctr) + 1;
  barrier(P, rank, world, epoch, SP_OPEN, err, 270);
  __shared__ float sred[32];
  const int nv = D / 8, v = threadIdx.x;
  for (int r = blockIdx.x; r < nrows; r += gridDim.x) {
    const int64_t g = (row0 + r) * (int64_t)D + 8 * v;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float ss = 0.f;
    if (v < nv) {
      for (int k = 0; k < world; ++k) {
        const int src = (rank + k) % world;        // stagger the peers each rank reads first
        float t[8];
        load8(reinterpret_cast<const bf16*>(P.buf[src]) + g, t);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += t[e];
      }
      bf16* xr = xs + (int64_t)r * D + 8 * v;
      float res[8];
      load8(xr, res);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        acc[e] = __bfloat162float(__float2bfloat16(acc[e] + res[e]));   // the stream is bf16
        ss += acc[e] * acc[e];
      }
      store8(xr, acc);
    }
    const float rstd = rsqrtf(block_sum(ss, sred) / (float)D + eps);
    if (v < nv) {
      float wf[8];
      load8(w + 8 * v, wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = acc[e] * rstd * wf[e];
      const uint4 o = make_uint4(pk2(acc[0], acc[1]), pk2(acc[2], acc[3]), pk2(acc[4], acc[5]), pk2(acc[6], acc[7]));
      for (int k = 0; k < world; ++k) {
        const int dst = (rank + k) % world;
        *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(H.p[dst]) + g) = o;
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned* done = ctr + 1;
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *done = 0u;
      for (int k = 0; k < world; ++k) st_release(P.flag[k] + SP_CLOSE * MAXR + rank, epoch);
      for (int k = 0; k < world; ++k) {
        const unsigned* f = P.flag[rank] + SP_CLOSE * MAXR + k;
        long long polls = 0;
        while ((int)(ld_acquire(f) - epoch) < 0) {
          if (++polls > kMaxPolls) {
            atomicExch(err, 271);
            break;
          }
          if (polls > 64) __nanosleep(128);
        }
      }
      *ctr = epoch;
      __threadfence();
    }
  }
}

// A bare cross-rank barrier on `slot` (one CTA).
__global__ void barrier_kernel(Peers P, int rank, int world, unsigned epoch, int slot, int* err) {
  barrier(P, rank, world, epoch, slot, err, 260 + slot);
}

}  // namespace symm

int symm_gather_bf16(void* const* bufs, int rank, int world, int64_t shard_len, bf16* dst, int blocks,
                     cudaStream_t s) {
  if (world > symm::MAXR || shard_len % 8) return -1;
  symm::Peers P{};
  for (int r = 0; r < world; ++r) P.buf[r] = bufs[r];
  symm::gather_kernel<<<blocks, 256, 0, s>>>(P, rank, world, shard_len, dst);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int symm_barrier(unsigned* const* flags, int rank, int world, unsigned epoch, int slot, int* err, cudaStream_t s) {
  if (world > symm::MAXR) return -1;
  symm::Peers P{};
  for (int r = 0; r < world; ++r) P.flag[r] = flags[r];
  symm::barrier_kernel<<<1, 32, 0, s>>>(P, rank, world, epoch, slot, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int symm_norm_coef(void* const* partials, unsigned* const* flags, int rank, int world, unsigned epoch, int nblocks,
                   float max_norm, float* norm_out, float* coef_out, int* err, cudaStream_t s) {
  symm::Peers P{};
  for (int r = 0; r < world && r < symm::MAXR; ++r) {
    P.buf[r] = partials[r];
    P.flag[r] = flags[r];
  }
  symm::norm_coef_kernel<<<1, 256, 0, s>>>(P, rank, world, epoch, nblocks, max_norm, norm_out, coef_out, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

static symm::Peers make_peers(void* const* bufs, unsigned* const* flags, int world) {
  symm::Peers P{};
  for (int r = 0; r < world && r < symm::MAXR; ++r) {
    P.buf[r] = bufs[r];
    P.flag[r] = flags[r];
  }
  return P;
}

int symm_allreduce_bf16(void* const* bufs, unsigned* const* flags, int rank, int world, unsigned* ctr, unsigned* done,
                        int64_t off, int64_t n, const bf16* residual, bf16* out, int* err, int sm_count,
                        cudaStream_t s) {
  if (world > symm::MAXR || n % 8) return -1;
  const int64_t n8 = n / 8;
  int blocks = (int)std::min<int64_t>((n8 + 255) / 256, (int64_t)sm_count * 2);
  if (blocks < 1) blocks = 1;
  symm::allreduce_kernel<<<blocks, 256, 0, s>>>(make_peers(bufs, flags, world), rank, world, ctr, done, off, n,
                                                residual, out, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int symm_rs_norm_ag(void* const* parts, void* const* gather, unsigned* const* flags, int rank, int world,
                    unsigned* ctr, int D, int64_t row0, int nrows, bf16* xs, const bf16* w, float eps, int* err,
                    int sm_count, cudaStream_t s) {
  if (world > symm::MAXR || D % 8 || D / 8 > 1024 || nrows < 0) return -1;
  symm::PeerBufs H{};
  for (int r = 0; r < world; ++r) H.p[r] = gather[r];
  const int threads = ((D / 8 + 31) / 32) * 32;
  const int blocks = std::max(1, std::min(nrows, sm_count * 2));
  symm::rs_norm_ag_kernel<<<blocks, threads, 0, s>>>(make_peers(parts, flags, world), H, rank, world, ctr, D, row0,
                                                     nrows, xs, w, eps, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int symm_rs_sumsq(void* const* bufs, unsigned* const* flags, int rank, int world, unsigned epoch, int64_t shard_off,
                  int64_t shard_len, float scale, float* shard_out, float* partial, int nblocks, int accumulate,
                  int* err, unsigned* done, int close_slot, cudaStream_t s) {
  if (world > symm::MAXR || shard_len % 4) return -1;
  if (close_slot >= 0 && done == nullptr) return -2;
  symm::rs_sumsq_kernel<<<nblocks, 256, 0, s>>>(make_peers(bufs, flags, world), rank, world, epoch, shard_off,
                                                shard_len, scale, shard_out, partial, accumulate, err, done,
                                                close_slot);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int symm_adamw_ag(void* const* bufs, unsigned* const* flags, int rank, int world, unsigned epoch, int64_t shard_off,
                  int64_t shard_len, const float* grad, float* master, float* m, float* v, float lr, float b1,
                  float b2, float eps, float wd, int step, const float* coef, unsigned* done, int* err, int sm_count,
                  cudaStream_t s) {
  if (world > symm::MAXR) return -1;
  const float bc1 = 1.f - powf(b1, (float)step), bc2 = 1.f - powf(b2, (float)step);
  int blocks = (int)std::min<int64_t>((shard_len + 255) / 256, (int64_t)sm_count * 4);
  if (blocks < 1) blocks = 1;
  symm::adamw_ag_kernel<<<blocks, 256, 0, s>>>(make_peers(bufs, flags, world), rank, world, epoch, shard_off,
                                               shard_len, grad, master, m, v, lr, b1, b2, eps, wd, bc1, bc2, coef,
                                               done, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// ---- IPC plumbing --------------------------------------------------------------------------
int symm_ipc_handle(void* ptr, unsigned char* out64) {
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return -1;
  memcpy(out64, &h, sizeof(h));
  return 0;
}

void* symm_ipc_open(const unsigned char* in64) {
  cudaIpcMemHandle_t h;
  memcpy(&h, in64, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return nullptr;
  return p;
}

void symm_ipc_close(void* p) { cudaIpcCloseMemHandle(p); }

}  // namespace trida
