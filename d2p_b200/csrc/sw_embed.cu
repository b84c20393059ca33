// sw_embed.cu -- the score producer in front of the alignment DP: for bf16
// embeddings X [B, L1, D] and Y [B, L2, D], scores[b] = scale * X[b] Y[b]^T
// in fp32 [B, L1, L2], the plane soft_sw and its relatives take (the
// reference builds it with an einsum outside its operators, docs/examples.md:
// 9-23, and takes it at d2p/sw.py:247).
//
// One CTA of 4 warps computes a 128 x 128 tile on the fifth-generation tensor
// cores: TMA brings the tile's rows of X and of Y into shared memory (D / 64
// chunks of 128 rows x 64 bf16, 128-byte swizzle, rows past the problem
// zero-filled), one thread issues D / 16 tcgen05.mma (kind::f16, bf16 x bf16
// -> fp32, M = N = 128, both operands K-major) into a 128-column TMEM
// accumulator and commits them to an mbarrier, and each warp reads its 32
// TMEM lanes (rows) back with tcgen05.ld into the operands' shared memory (the
// tile as four 32-column boxes, 128-byte swizzle: conflict-free 16-byte
// stores), which leaves by four TMA stores (direct stores when the rows are
// not whole 16-byte units).  Every wait is
// bounded; a tile whose copy or product did not arrive in time is recomputed
// by the CTA's CUDA cores from global memory and counted in the status word,
// after bounded waits for what was in flight, and the TMEM is freed on every
// path.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#include "../../include/d2p_b200.h"
#include "sw_common.cuh"
#include "sw_internal.h"

namespace d2pb {
namespace emb {

constexpr int kTile = 128;                       // rows and columns of an output tile
constexpr int kKC = 64;                          // bf16 per K chunk: one 128-byte swizzle row
constexpr int kMaxD = 256;
constexpr int kChunkBytes = kTile * kKC * 2;     // 16 KB
constexpr int kThreads = 128;
constexpr int kSpin = 1 << 22;                   // bounded waits

constexpr int kStage = 4 * kChunkBytes;          // the fp32 output tile staged for its TMA store (64 KB)
// operand chunks (or the staged output tile, which reuses them), then the
// barriers; at least 64 KB, so that no more than three CTAs (3 x 128 of an
// SM's 512 TMEM columns) share an SM and an allocation never waits
__host__ __device__ inline int bars_offset(int D) {
    const int a = 2 * (D / kKC) * kChunkBytes;
    return a > kStage ? a : kStage;
}
__host__ __device__ inline size_t smem_bytes(int D) { return (size_t)bars_offset(D) + 1024 + 64; }

__device__ __forceinline__ unsigned smem_u32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }

__device__ __forceinline__ bool bar_wait(unsigned bar, unsigned parity) {
    for (int it = 0; it < kSpin; ++it) {
        unsigned done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(bar), "r"(parity)
            : "memory");
        if (done) return true;
        if (it > 64) __nanosleep(32);
    }
    return false;
}

// shared-memory matrix descriptor of a K-major, 128-byte-swizzled operand
// chunk (rows of 128 bytes, 8-row groups 1024 bytes apart), sm_100 form
__device__ __forceinline__ uint64_t umma_desc(unsigned saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// instruction descriptor: fp32 accumulator, bf16 A and B, both K-major, N = M = 128
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTile >> 3) << 17) |
                            ((uint32_t)(kTile >> 4) << 24);

__global__ void __launch_bounds__(kThreads) embed_scores_kernel(const __grid_constant__ CUtensorMap tmX,
                                                                const __grid_constant__ CUtensorMap tmY,
                                                                const __grid_constant__ CUtensorMap tmS, int tma_out,
                                                                const __nv_bfloat16* __restrict__ X,
                                                                const __nv_bfloat16* __restrict__ Y,
                                                                float* __restrict__ S, int L1, int L2, int D,
                                                                float scale, int* status) {
    extern __shared__ uint8_t raw[];
    const unsigned r0 = smem_u32(raw);
    const unsigned sbase = (r0 + 1023u) & ~1023u;           // TMA / swizzle atoms want 1024-byte alignment
    uint8_t* gbase = raw + (sbase - r0);
    const int nK = D / kKC;
    const unsigned sA = sbase, sB = sbase + nK * kChunkBytes;
    unsigned long long* bars = reinterpret_cast<unsigned long long*>(gbase + bars_offset(D));
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);
    int* okflag = reinterpret_cast<int*>(bars + 3);
    const unsigned barT = smem_u32(&bars[0]), barM = smem_u32(&bars[1]);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * kTile, m0 = blockIdx.y * kTile, b = blockIdx.z;

    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(barT) : "memory");
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(barM) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        *okflag = 0;
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                     "r"(kTile)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tslot;

    if (tid == 0) {
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(barT), "r"(2 * nK * kChunkBytes)
                     : "memory");
        for (int kc = 0; kc < nK; ++kc) {
            asm volatile(
                "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
                "%4}], [%5];" ::"r"(sA + kc * kChunkBytes),
                "l"((unsigned long long)&tmX), "r"(kc * kKC), "r"(m0), "r"(b), "r"(barT)
                : "memory");
            asm volatile(
                "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
                "%4}], [%5];" ::"r"(sB + kc * kChunkBytes),
                "l"((unsigned long long)&tmY), "r"(kc * kKC), "r"(n0), "r"(b), "r"(barT)
                : "memory");
        }
        if (bar_wait(barT, 0)) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            for (int kc = 0; kc < nK; ++kc) {
#pragma unroll
                for (int kk = 0; kk < kKC / 16; ++kk) {   // K = 16 per instruction: 32 bytes along the row
                    const uint64_t da = umma_desc(sA + kc * kChunkBytes + kk * 32);
                    const uint64_t db = umma_desc(sB + kc * kChunkBytes + kk * 32);
                    const uint32_t acc = (kc | kk) != 0;
                    asm volatile(
                        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
                        "l"(da), "l"(db), "r"(kIdesc), "r"(acc)
                        : "memory");
                }
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(barM)
                         : "memory");
            *okflag = 1;
        }
    }
    __syncthreads();
    const bool issued = *okflag != 0;
    const bool done = issued && bar_wait(barM, 0);
    const bool all = __syncthreads_and(done);   // one decision for the CTA
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int row = m0 + 32 * warp + lane;
    float* srow = S + ((size_t)b * L1 + (row < L1 ? row : 0)) * L2;
    if (all) {
#pragma unroll 1
        for (int c = 0; c < kTile / 32; ++c) {
            uint32_t v[32];
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
                "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
                : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                  "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                  "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
                  "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
                  "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
                : "r"(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(32 * c)));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            const int col0 = n0 + 32 * c;
            if (tma_out) {   // into box c of the staged tile: 128-byte rows, 16-byte chunks swizzled by row
                const int r = 32 * warp + lane;
                uint8_t* rowp = gbase + c * kChunkBytes + r * 128;
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    *reinterpret_cast<float4*>(rowp + ((q ^ (r & 7)) << 4)) =
                        make_float4(scale * __uint_as_float(v[4 * q]), scale * __uint_as_float(v[4 * q + 1]),
                                    scale * __uint_as_float(v[4 * q + 2]), scale * __uint_as_float(v[4 * q + 3]));
            } else if (row < L1) {
                if (col0 + 32 <= L2 && (L2 & 3) == 0) {
                    float4* dst = reinterpret_cast<float4*>(srow + col0);
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        dst[q] = make_float4(scale * __uint_as_float(v[4 * q]), scale * __uint_as_float(v[4 * q + 1]),
                                             scale * __uint_as_float(v[4 * q + 2]),
                                             scale * __uint_as_float(v[4 * q + 3]));
                } else {
#pragma unroll
                    for (int q = 0; q < 32; ++q)
                        if (col0 + q < L2) srow[col0 + q] = scale * __uint_as_float(v[q]);
                }
            }
        }
        if (tma_out) {   // four 32-column boxes; rows and columns past the problem are clipped by the copy
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncthreads();
            if (tid == 0) {
#pragma unroll
                for (int c = 0; c < kTile / 32; ++c)
                    asm volatile(
                        "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
                            (unsigned long long)&tmS),
                        "r"(n0 + 32 * c), "r"(m0), "r"(b), "r"(sbase + c * kChunkBytes)
                        : "memory");
                asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
            }
        }
    } else {
        // a copy or the product did not arrive in time: count it, wait (bounded)
        // for what is in flight, and compute the tile on the CUDA cores
        if (tid == 0 && status) atomicAdd(status, 1);
        bar_wait(barT, 0);
        if (issued) bar_wait(barM, 0);
        if (row < L1) {
            const __nv_bfloat16* xr = X + ((size_t)b * L1 + row) * D;
            for (int j = n0; j < min(n0 + kTile, L2); ++j) {
                const __nv_bfloat16* yr = Y + ((size_t)b * L2 + j) * D;
                float acc = 0.f;
                for (int d = 0; d < D; ++d) acc = fmaf(__bfloat162float(xr[d]), __bfloat162float(yr[d]), acc);
                srow[j] = scale * acc;
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTile) : "memory");
}

// G[b] = bf16(scale * g[b] * P[b]): the gradient of the scores for a loss
// that reaches only the values, in the operand type of the embeddings'
// gradient GEMMs (8 elements per thread: 32 bytes read, 16 written)
__global__ void grad_scores_bf16_kernel(const float* __restrict__ P, const float* __restrict__ g, float scale,
                                        size_t plane, size_t n8, __nv_bfloat16* __restrict__ G) {
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n8; e += (size_t)gridDim.x * blockDim.x) {
        const size_t i = e * 8;
        const float s = scale * __ldg(g + i / plane);
        const float4 a = __ldcs(reinterpret_cast<const float4*>(P + i));
        const float4 c = __ldcs(reinterpret_cast<const float4*>(P + i + 4));
        __nv_bfloat162 o[4] = {__floats2bfloat162_rn(s * a.x, s * a.y), __floats2bfloat162_rn(s * a.z, s * a.w),
                               __floats2bfloat162_rn(s * c.x, s * c.y), __floats2bfloat162_rn(s * c.z, s * c.w)};
        *reinterpret_cast<uint4*>(G + i) = *reinterpret_cast<uint4*>(o);
    }
}
// the same, one element per thread (planes that are not whole 8-element units)
__global__ void grad_scores_bf16_scalar_kernel(const float* __restrict__ P, const float* __restrict__ g, float scale,
                                               size_t plane, size_t n, __nv_bfloat16* __restrict__ G) {
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x)
        G[e] = __float2bfloat16_rn(scale * __ldg(g + e / plane) * __ldcs(P + e));
}

}  // namespace emb

namespace {
PFN_cuTensorMapEncodeTiled_v12000 embed_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

// [B][L][D] bf16 as a 3-D tensor (D, rows, problem), boxes of 64 x 128 x 1
// with the 128-byte swizzle; rows past L read as zeros
// the fp32 score plane [B][L1][L2] (L2 a multiple of 4) as a 3-D tensor, boxes
// of 32 columns x 128 rows with the 128-byte swizzle (the staged tile's layout)
bool scores_tensor_map(CUtensorMap* tm, float* base, int B, int L1, int L2) {
    auto fn = embed_encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)L2, (cuuint64_t)L1, (cuuint64_t)B};
    const cuuint64_t strides[2] = {(cuuint64_t)L2 * 4, (cuuint64_t)L1 * L2 * 4};
    const cuuint32_t box[3] = {32, (cuuint32_t)emb::kTile, 1};
    const cuuint32_t es[3] = {1, 1, 1};
    return fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool embed_tensor_map(CUtensorMap* tm, const void* base, int B, int L, int D) {
    auto fn = embed_encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)L, (cuuint64_t)B};
    const cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)L * D * 2};
    const cuuint32_t box[3] = {(cuuint32_t)emb::kKC, (cuuint32_t)emb::kTile, 1};
    const cuuint32_t es[3] = {1, 1, 1};
    return fn(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

}  // namespace d2pb

using namespace d2pb;

extern "C" {

int d2p_embed_scores(const void* x, const void* y, int B, int L1, int L2, int D, float scale, float* scores,
                     int* status, void* stream) {
    if (B < 0 || L1 < 0 || L2 < 0 || D < 0) return D2P_ERR_INVALID_ARGUMENT;
    if (B == 0 || L1 == 0 || L2 == 0) return D2P_OK;
    if (!x || !y || !scores) return D2P_ERR_INVALID_ARGUMENT;
    if (D == 0 || D % emb::kKC != 0) return D2P_ERR_INVALID_ARGUMENT;   // pad the embeddings to a multiple of 64
    if (D > emb::kMaxD || B > 65535) return D2P_ERR_TOO_LARGE;
    if (((uintptr_t)x | (uintptr_t)y) & 15) return D2P_ERR_INVALID_ARGUMENT;
    CUtensorMap tmX, tmY, tmS;
    if (!embed_tensor_map(&tmX, x, B, L1, D) || !embed_tensor_map(&tmY, y, B, L2, D)) return D2P_ERR_INVALID_ARGUMENT;
    // the staged tile leaves by TMA when the rows are whole 16-byte units; else by direct stores
    const int tma_out = (L2 % 4 == 0 && ((uintptr_t)scores & 15) == 0 && scores_tensor_map(&tmS, scores, B, L1, L2));
    if (!tma_out) memset(&tmS, 0, sizeof(tmS));
    static DeviceSetup setup;
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    int rc = device_setup(setup, dev, [] {
        return (int)cudaFuncSetAttribute(emb::embed_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)emb::smem_bytes(emb::kMaxD));
    }, &sms);
    if (rc) return rc;
    const dim3 grid((L2 + emb::kTile - 1) / emb::kTile, (L1 + emb::kTile - 1) / emb::kTile, B);
    emb::embed_scores_kernel<<<grid, emb::kThreads, emb::smem_bytes(D), (cudaStream_t)stream>>>(
        tmX, tmY, tmS, tma_out, (const __nv_bfloat16*)x, (const __nv_bfloat16*)y, scores, L1, L2, D, scale, status);
    return (int)cudaGetLastError();
}

int d2p_embed_grad_scores(const float* marginals, const float* grad_value, int B, int L1, int L2, float scale,
                          void* grad_scores_bf16, void* stream) {
    if (B < 0 || L1 < 0 || L2 < 0) return D2P_ERR_INVALID_ARGUMENT;
    const size_t plane = (size_t)L1 * L2, n = plane * (size_t)B;
    if (n == 0) return D2P_OK;
    if (!marginals || !grad_value || !grad_scores_bf16) return D2P_ERR_INVALID_ARGUMENT;
    static DeviceSetup setup;
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    int rc = device_setup(setup, dev, [] { return 0; }, &sms);
    if (rc) return rc;
    const int threads = 256;
    const bool vec = plane % 8 == 0 && ((((uintptr_t)marginals | (uintptr_t)grad_scores_bf16) & 15) == 0);
    const size_t units = vec ? n / 8 : n;
    const size_t want = (units + threads - 1) / threads;
    const int blocks = (int)(want < (size_t)sms * 16 ? want : (size_t)sms * 16);
    if (vec)
        emb::grad_scores_bf16_kernel<<<blocks, threads, 0, (cudaStream_t)stream>>>(
            marginals, grad_value, scale, plane, units, (__nv_bfloat16*)grad_scores_bf16);
    else
        emb::grad_scores_bf16_scalar_kernel<<<blocks, threads, 0, (cudaStream_t)stream>>>(
            marginals, grad_value, scale, plane, units, (__nv_bfloat16*)grad_scores_bf16);
    return (int)cudaGetLastError();
}

}  // extern "C"
