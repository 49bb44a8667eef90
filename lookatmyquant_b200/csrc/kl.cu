// The KL probe's head on tcgen05: LM-head logits, log-softmax and the KL to the reference distribution in one pass
// over the vocabulary, without writing logits.
//
// Reference: compiler.py:176-187 (`measure`): ref_lp = log_softmax(model(held).logits.float()) once; per probe
// lp = log_softmax(model(held).logits.float()) and KL = Σ_t w_t·Σ_v exp(lr_tv)·(lr_tv − lp_tv) / Σ_t w_t. The model's
// lm_head is a bf16 GEMM whose logits are bf16 (rounded from an fp32 accumulation), then cast to fp32.
//
// With z the logits of a position, lse = log Σ_v exp(z_v), p the reference distribution and z_ref, lse_ref its logits:
//   KL_t = Σ_v p_v·(z_ref,v − lse_ref − z_v + lse) = A_t − B_t + (lse_t − lse_ref,t)·P_t,
//   A_t = Σ_v p_v·z_ref,v,  B_t = Σ_v p_v·z_v,  P_t = Σ_v p_v.
// Three passes of one kernel, each a tcgen05 GEMM Z = H·Eᵀ (H: positions x d, E: V x d, both bf16 and K-major; tiles
// of 128 positions x 256 vocabulary entries, fp32 in TMEM, rounded to bf16 as the reference's lm_head rounds) with a
// per-row epilogue over the vocabulary:
//   kModeLse    online max and sum of exponentials        → lse (the reference's, once);
//   kModeRef    p = exp(z − lse_ref) written (fp32), A and P accumulated    (once per held set);
//   kModeProbe  p read, online max/sum and B accumulated  → lse and B (every probe).
// Work units are (vocabulary range, block of 128 positions); each writes per-row partials, which a small kernel
// combines in a fixed order (deterministic). The probe pass of the unquantized model reproduces A exactly, so its KL
// is exactly zero, as the reference's floor is.
//
// Warp roles (320 threads): warp 0 issues TMA loads (4-stage ring of 64-wide K slices of H and E), warp 1 issues the
// MMAs into two TMEM accumulators (256 columns each), warps 2-9 drain a finished accumulator (two warps per TMEM lane
// quadrant, 128 columns each) while the next one fills.
#include <algorithm>
#include <mutex>

#include <cuda.h>
#include <cuda_bf16.h>

#include "lamq_common.cuh"
#include "sm100.cuh"

namespace lamq {
namespace {

using namespace sm100;

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int kEpiWarps = 8, kThreads = (2 + kEpiWarps) * 32;
constexpr uint32_t kTmemCols = 512;
constexpr size_t kSmemBytes = 1024 + STAGES * STAGE_BYTES + 256;
constexpr int kVSplit = 16;  // vocabulary ranges per block of positions
constexpr int kModeLse = 0, kModeRef = 1, kModeProbe = 2;
constexpr float kLog2e = 1.4426950408889634f;

struct KLParams {
    int64_t ntok;
    int d, V;
    int kblocks, nvb, vb_per_unit, npb;
    int64_t units;
    int mode;
    float *p;              // ntok x V fp32 reference distribution (written in kModeRef, read in kModeProbe)
    int64_t ldp;
    const float *lse_ref;  // ntok (kModeRef)
    float *part_m, *part_s;  // ntok x kVSplit x 2
    double *part_b;
    int *status;
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float4 ld_stream(const float *p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void st_stream(float *p, float4 v) {
    asm volatile("st.global.L1::no_allocate.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z),
                 "f"(v.w)
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

// Unit u: vocabulary range u / npb (blocks vr·vb_per_unit ...), position block u % npb — consecutive units share E.
__device__ __forceinline__ void unit_of(int64_t u, const KLParams &p, int &pb, int &vb0, int &vb1, int &vr) {
    vr = (int)(u / p.npb);
    pb = (int)(u % p.npb);
    vb0 = vr * p.vb_per_unit;
    vb1 = min(p.nvb, vb0 + p.vb_per_unit);
}

__global__ void __launch_bounds__(kThreads, 1)
    kl_head_kernel(const __grid_constant__ CUtensorMap mapH, const __grid_constant__ CUtensorMap mapE, KLParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 5);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES);
    const uint32_t tfull0 = smem_u32(bars + 2 * STAGES), tempty0 = smem_u32(bars + 2 * STAGES + 2);
    const uint32_t drain = smem_u32(bars + 2 * STAGES + 4);
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull0 + 8 * a, 1);
            mbar_init(tempty0 + 8 * a, kEpiWarps * 32);
        }
        mbar_init(drain, 1);
        fence_mbar_init();
        prefetch_tmap(&mapH);
        prefetch_tmap(&mapE);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_holder), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0) {
        if (lane == 0) {  // ---- TMA producer
            int stage = 0;
            uint32_t phase = 0;
            int64_t issued = 0;
            bool ok = true;
            for (int64_t u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
                int pb, vb0, vb1, vr;
                unit_of(u, p, pb, vb0, vb1, vr);
                for (int vb = vb0; ok && vb < vb1; ++vb) {
                    for (int kb = 0; kb < p.kblocks; ++kb) {
                        if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, p.status)) {
                            ok = false;
                            break;
                        }
                        const uint32_t fb = full0 + 8 * stage;
                        mbar_expect_tx(fb, STAGE_BYTES);
                        const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES), sb = sa + A_BYTES;
                        tma_load_2d(sa, &mapH, kb * BK, pb * BM, fb);
                        tma_load_2d(sb, &mapE, kb * BK, vb * BN, fb);
                        ++issued;
                        if (++stage == STAGES) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
            }
            if (!ok) {  // error path: let the copies in flight land before the CTA exits
                const int64_t outstanding = issued < STAGES ? issued : STAGES;
                for (int64_t i = issued - outstanding; i < issued; ++i) {
                    const int s = (int)(i % STAGES);
                    const uint32_t ph = (uint32_t)((i / STAGES) & 1);
                    const unsigned long long t0 = globaltimer();
                    while (!mbar_try_wait(full0 + 8 * s, ph) && globaltimer() - t0 < kWaitTimeoutNs) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // ---- MMA issuer
            const uint32_t idesc = idesc_bf16_f32(BM, BN, false, false);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t uses[2] = {0, 0};
            int acc = 0;
            bool ok = true;
            for (int64_t u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
                int pb, vb0, vb1, vr;
                unit_of(u, p, pb, vb0, vb1, vr);
                for (int vb = vb0; ok && vb < vb1; ++vb) {
                    if (!mbar_wait(tempty0 + 8 * acc, (uses[acc] & 1) ^ 1, p.status)) {
                        ok = false;
                        break;
                    }
                    ++uses[acc];
                    tc_fence_after();
                    const uint32_t dt = tmem + acc * BN;
                    for (int kb = 0; kb < p.kblocks; ++kb) {
                        if (!mbar_wait(full0 + 8 * stage, phase, p.status)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES), sb = sa + A_BYTES;
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk) {
                            // K-major, 128-byte swizzle: 16 elements of K are 32 bytes along each 128-byte row
                            const uint64_t ad = smem_desc_sw128(sa + kk * 32, 16, 1024);
                            const uint64_t bd = smem_desc_sw128(sb + kk * 32, 16, 1024);
                            mma_f16_ss(dt, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                        }
                        mma_commit(empty0 + 8 * stage);
                        if (++stage == STAGES) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                    if (!ok) break;
                    mma_commit(tfull0 + 8 * acc);
                    acc ^= 1;
                }
            }
            mma_commit(drain);
            const unsigned long long t0 = globaltimer();
            while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < kWaitTimeoutNs) {
            }
        }
    } else {  // ---- epilogue: warp w reads TMEM lanes 32·(w % 4).., columns 128·((w − 2) / 4)..
        const int q = warp & 3, half = (warp - 2) >> 2;
        uint32_t uses[2] = {0, 0};
        int acc = 0;
        for (int64_t u = blockIdx.x; u < p.units; u += gridDim.x) {
            int pb, vb0, vb1, vr;
            unit_of(u, p, pb, vb0, vb1, vr);
            const int64_t row = (int64_t)pb * BM + 32 * q + lane;
            const bool live = row < p.ntok;
            const float lref = (p.mode == kModeRef && live) ? p.lse_ref[row] : 0.f;
            float m = -INFINITY, s = 0.f;
            double b = 0.0, pa = 0.0;  // B (or A) and P
            bool ok = true;
            for (int vb = vb0; vb < vb1; ++vb) {
                if (!mbar_wait(tfull0 + 8 * acc, uses[acc] & 1, p.status)) {
                    ok = false;
                    break;
                }
                ++uses[acc];
                tc_fence_after();
                const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16) + acc * BN + 128 * half;
                float bsum = 0.f, psum = 0.f;
#pragma unroll 1
                for (int c = 0; c < 128 / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld32(tbase + c * 32, r);
                    tmem_ld_wait();
                    const int v0 = vb * BN + 128 * half + 32 * c;
                    float z[32];
#pragma unroll
                    for (int e = 0; e < 32; ++e) {
                        // the lm_head's bf16 logits; vocabulary entries past V do not exist
                        const float zz = __bfloat162float(__float2bfloat16_rn(__uint_as_float(r[e])));
                        z[e] = (v0 + e < p.V) ? zz : -INFINITY;
                    }
                    if (p.mode != kModeRef) {
                        float cm = m;
#pragma unroll
                        for (int e = 0; e < 32; ++e) cm = fmaxf(cm, z[e]);
                        if (cm != -INFINITY) {  // a chunk wholly past V leaves the running values alone
                            float cs = 0.f;
#pragma unroll
                            for (int e = 0; e < 32; ++e) cs += ex2((z[e] - cm) * kLog2e);
                            s = (m == -INFINITY ? 0.f : s * ex2((m - cm) * kLog2e)) + cs;
                            m = cm;
                        }
                    }
                    if (p.mode != kModeLse && live) {
                        float *prow = p.p + row * p.ldp + v0;
#pragma unroll
                        for (int e = 0; e < 32; e += 4) {
                            float4 pv;
                            if (p.mode == kModeRef) {
                                pv.x = (v0 + e + 0 < p.V) ? expf(z[e + 0] - lref) : 0.f;
                                pv.y = (v0 + e + 1 < p.V) ? expf(z[e + 1] - lref) : 0.f;
                                pv.z = (v0 + e + 2 < p.V) ? expf(z[e + 2] - lref) : 0.f;
                                pv.w = (v0 + e + 3 < p.V) ? expf(z[e + 3] - lref) : 0.f;
                                if (v0 + e + 3 < p.V) {
                                    st_stream(prow + e, pv);
                                } else {
                                    if (v0 + e + 0 < p.V) prow[e + 0] = pv.x;
                                    if (v0 + e + 1 < p.V) prow[e + 1] = pv.y;
                                    if (v0 + e + 2 < p.V) prow[e + 2] = pv.z;
                                }
                                psum += (pv.x + pv.y) + (pv.z + pv.w);
                            } else {
                                if (v0 + e + 3 < p.V) {
                                    pv = ld_stream(prow + e);
                                } else {
                                    pv.x = (v0 + e + 0 < p.V) ? prow[e + 0] : 0.f;
                                    pv.y = (v0 + e + 1 < p.V) ? prow[e + 1] : 0.f;
                                    pv.z = (v0 + e + 2 < p.V) ? prow[e + 2] : 0.f;
                                    pv.w = 0.f;
                                }
                            }
                            // Σ p·z (zero p past V multiplies −inf: skip those)
                            if (v0 + e + 0 < p.V) bsum = fmaf(pv.x, z[e + 0], bsum);
                            if (v0 + e + 1 < p.V) bsum = fmaf(pv.y, z[e + 1], bsum);
                            if (v0 + e + 2 < p.V) bsum = fmaf(pv.z, z[e + 2], bsum);
                            if (v0 + e + 3 < p.V) bsum = fmaf(pv.w, z[e + 3], bsum);
                        }
                    }
                }
                tc_fence_before();
                mbar_arrive(tempty0 + 8 * acc);
                acc ^= 1;
                b += (double)bsum;
                pa += (double)psum;
            }
            if (!ok) break;
            if (live) {
                const int64_t slot = (row * kVSplit + vr) * 2 + half;
                p.part_m[slot] = m;
                p.part_s[slot] = (p.mode == kModeRef) ? (float)pa : s;
                p.part_b[slot] = b;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// Per row: the partials of the ranges and halves in a fixed order.
//   kModeLse:   lse → lse_out
//   kModeRef:   A → stat_a, P → stat_p
//   kModeProbe: KL_t = A − B + (lse − lse_ref)·P → kl_pos; Σ w·KL and Σ w → sums[0], sums[1]
__global__ void kl_combine_kernel(int mode, int64_t ntok, int nranges, const float *__restrict__ part_m,
                                  const float *__restrict__ part_s, const double *__restrict__ part_b, float *lse_out,
                                  double *stat_a, double *stat_p, const float *__restrict__ lse_ref,
                                  const float *__restrict__ w, float *kl_pos, double *sums) {
    __shared__ double red[2][256];
    double wk = 0.0, ws = 0.0;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < ntok; t += (int64_t)gridDim.x * blockDim.x) {
        const float *pm = part_m + t * kVSplit * 2;
        const float *ps = part_s + t * kVSplit * 2;
        const double *pbv = part_b + t * kVSplit * 2;
        double B = 0.0, P = 0.0;
        float M = -INFINITY;
        for (int i = 0; i < nranges * 2; ++i) {
            B += pbv[i];
            if (mode == kModeRef) P += (double)ps[i];
            else M = fmaxf(M, pm[i]);
        }
        if (mode == kModeRef) {
            stat_a[t] = B;
            stat_p[t] = P;
            continue;
        }
        float S = 0.f;
        for (int i = 0; i < nranges * 2; ++i)
            if (pm[i] != -INFINITY) S += ps[i] * ex2((pm[i] - M) * kLog2e);
        const float lse = M + logf(S);
        if (mode == kModeLse) {
            lse_out[t] = lse;
            continue;
        }
        const double kl = stat_a[t] - B + ((double)lse - (double)lse_ref[t]) * stat_p[t];
        kl_pos[t] = (float)kl;
        const double wt = w ? (double)w[t] : 1.0;
        wk += wt * kl;
        ws += wt;
    }
    if (mode != kModeProbe) return;
    red[0][threadIdx.x] = wk;
    red[1][threadIdx.x] = ws;
    __syncthreads();
    for (int h = blockDim.x / 2; h > 0; h >>= 1) {
        if (threadIdx.x < h) {
            red[0][threadIdx.x] += red[0][threadIdx.x + h];
            red[1][threadIdx.x] += red[1][threadIdx.x + h];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        sums[2 * blockIdx.x] = red[0][0];
        sums[2 * blockIdx.x + 1] = red[1][0];
    }
}

__global__ void fill_kernel(float *x, int64_t n, float v) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) x[e] = v;
}

// The final sums over the combine blocks, in order.
__global__ void kl_total_kernel(const double *sums, int nblocks, double *out) {
    double a = 0.0, b = 0.0;
    for (int i = 0; i < nblocks; ++i) {
        a += sums[2 * i];
        b += sums[2 * i + 1];
    }
    out[0] = a / b;
    out[1] = a;
    out[2] = b;
}

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
    static std::once_flag once;
    static EncodeTiled fn = nullptr;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(ptr);
    });
    return fn;
}

// rows x d bf16, K (d) contiguous: boxes of 64 x box_rows, 128-byte swizzle (the K-major operand layout).
int make_kmajor_map(CUtensorMap *m, const void *base, int64_t rows, int d, int64_t ld, int box_rows) {
    EncodeTiled enc = encode_fn();
    if (enc == nullptr) {
        set_error("lamq_kl_head: cuTensorMapEncodeTiled is unavailable");
        return LAMQ_ERR_CUDA;
    }
    cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("lamq_kl_head: cuTensorMapEncodeTiled failed (%d)", (int)r);
        return LAMQ_ERR_INVALID;
    }
    return LAMQ_OK;
}

int num_sms() {
    static int sms = 0;
    if (sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    return sms;
}

constexpr int kCombineBlocks = 148;

struct KLLayout {
    size_t m, s, b, sums, total;
};

KLLayout kl_layout(int64_t ntok) {
    auto up = [](size_t x) { return (x + 255) / 256 * 256; };
    KLLayout l{};
    const size_t parts = (size_t)ntok * kVSplit * 2;
    l.m = up(parts * sizeof(float));
    l.s = up(parts * sizeof(float));
    l.b = up(parts * sizeof(double));
    l.sums = up(2 * kCombineBlocks * sizeof(double));
    l.total = l.m + l.s + l.b + l.sums;
    return l;
}

int run_pass(int mode, const uint16_t *H, int64_t ldh, int64_t ntok, int d, const uint16_t *E, int64_t lde, int V,
             float *pdist, int64_t ldp, const float *lse_ref, void *workspace, int *status, cudaStream_t s,
             KLLayout &l, float **pm, float **ps, double **pbv, double **sums) {
    CUtensorMap mh, me;
    int st = make_kmajor_map(&mh, H, ntok, d, ldh, BM);
    if (st) return st;
    st = make_kmajor_map(&me, E, V, d, lde, BN);
    if (st) return st;
    l = kl_layout(ntok);
    uint8_t *base = reinterpret_cast<uint8_t *>(workspace);
    *pm = reinterpret_cast<float *>(base);
    *ps = reinterpret_cast<float *>(base + l.m);
    *pbv = reinterpret_cast<double *>(base + l.m + l.s);
    *sums = reinterpret_cast<double *>(base + l.m + l.s + l.b);
    KLParams p{};
    p.ntok = ntok;
    p.d = d;
    p.V = V;
    p.kblocks = (d + BK - 1) / BK;
    p.nvb = (V + BN - 1) / BN;
    p.vb_per_unit = (p.nvb + kVSplit - 1) / kVSplit;
    p.npb = (int)((ntok + BM - 1) / BM);
    const int nranges = (p.nvb + p.vb_per_unit - 1) / p.vb_per_unit;
    p.units = (int64_t)nranges * p.npb;
    p.mode = mode;
    p.p = pdist;
    p.ldp = ldp;
    p.lse_ref = lse_ref;
    p.part_m = *pm;
    p.part_s = *ps;
    p.part_b = *pbv;
    p.status = status;
    // ranges past the last one hold no partials: mark them empty so the combine skips them
    cudaError_t e = cudaMemsetAsync(*pbv, 0, l.b, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(*ps, 0, l.s, s);
    if (e == cudaSuccess) e = smem_limit_once((const void *)kl_head_kernel, (int)kSmemBytes);
    if (e != cudaSuccess) {
        set_error("lamq_kl_head: %s", cudaGetErrorString(e));
        return LAMQ_ERR_CUDA;
    }
    // part_m: −inf everywhere, so absent ranges drop out of the max
    fill_kernel<<<148, 256, 0, s>>>(*pm, (int64_t)ntok * kVSplit * 2, -INFINITY);
    LAMQ_CHECK_LAUNCH("lamq_kl_head fill");
    const int64_t grid = std::min<int64_t>(p.units, num_sms());
    kl_head_kernel<<<(unsigned)grid, kThreads, kSmemBytes, s>>>(mh, me, p);
    LAMQ_CHECK_LAUNCH("lamq_kl_head");
    return LAMQ_OK;
}

int check_args(const char *fn, const uint16_t *H, int64_t ldh, int64_t ntok, int d, const uint16_t *E, int64_t lde,
               int V) {
    LAMQ_REQUIRE(ntok > 0 && d > 0 && V > 0, "%s: bad shape", fn);
    LAMQ_REQUIRE(H && E, "%s: null pointer", fn);
    LAMQ_REQUIRE(d % 8 == 0 && ldh % 8 == 0 && lde % 8 == 0 && ldh >= d && lde >= d,
                 "%s: d and leading dimensions must be multiples of 8 (16-byte rows for TMA)", fn);
    LAMQ_REQUIRE(((uintptr_t)H % 16) == 0 && ((uintptr_t)E % 16) == 0, "%s: operands not 16-byte aligned", fn);
    return LAMQ_OK;
}

}  // namespace
}  // namespace lamq

using namespace lamq;

extern "C" size_t lamq_kl_workspace_size(int64_t ntok) { return ntok <= 0 ? 0 : kl_layout(ntok).total; }

extern "C" int lamq_kl_reference(const uint16_t *H, int64_t ldh, int64_t ntok, int d, const uint16_t *E, int64_t lde,
                                 int V, float *pdist, int64_t ldp, float *lse_ref, double *stat_a, double *stat_p,
                                 void *workspace, size_t workspace_bytes, int *status, lamq_stream_t stream) {
    int st = check_args("lamq_kl_reference", H, ldh, ntok, d, E, lde, V);
    if (st) return st;
    LAMQ_REQUIRE(pdist && lse_ref && stat_a && stat_p && workspace && status, "lamq_kl_reference: null pointer");
    LAMQ_REQUIRE(ldp >= V && ldp % 4 == 0 && ((uintptr_t)pdist % 16) == 0,
                 "lamq_kl_reference: the distribution's rows must be 16-byte aligned with ldp >= V");
    LAMQ_REQUIRE(workspace_bytes >= lamq_kl_workspace_size(ntok), "lamq_kl_reference: workspace too small");
    cudaStream_t s = (cudaStream_t)stream;
    KLLayout l;
    float *pm, *ps;
    double *pbv, *sums;
    st = run_pass(kModeLse, H, ldh, ntok, d, E, lde, V, nullptr, 0, nullptr, workspace, status, s, l, &pm, &ps, &pbv,
                  &sums);
    if (st) return st;
    const int nranges = kVSplit;
    kl_combine_kernel<<<kCombineBlocks, 256, 0, s>>>(kModeLse, ntok, nranges, pm, ps, pbv, lse_ref, nullptr, nullptr,
                                                     nullptr, nullptr, nullptr, sums);
    LAMQ_CHECK_LAUNCH("lamq_kl_reference combine");
    st = run_pass(kModeRef, H, ldh, ntok, d, E, lde, V, pdist, ldp, lse_ref, workspace, status, s, l, &pm, &ps, &pbv,
                  &sums);
    if (st) return st;
    kl_combine_kernel<<<kCombineBlocks, 256, 0, s>>>(kModeRef, ntok, nranges, pm, ps, pbv, nullptr, stat_a, stat_p,
                                                     nullptr, nullptr, nullptr, sums);
    LAMQ_CHECK_LAUNCH("lamq_kl_reference combine");
    return LAMQ_OK;
}

extern "C" int lamq_kl_head(const uint16_t *H, int64_t ldh, int64_t ntok, int d, const uint16_t *E, int64_t lde, int V,
                            const float *pdist, int64_t ldp, const float *lse_ref, const double *stat_a,
                            const double *stat_p, const float *w, float *kl_pos, double *kl_out, void *workspace,
                            size_t workspace_bytes, int *status, lamq_stream_t stream) {
    int st = check_args("lamq_kl_head", H, ldh, ntok, d, E, lde, V);
    if (st) return st;
    LAMQ_REQUIRE(pdist && lse_ref && stat_a && stat_p && kl_pos && kl_out && workspace && status,
                 "lamq_kl_head: null pointer");
    LAMQ_REQUIRE(ldp >= V && ldp % 4 == 0 && ((uintptr_t)pdist % 16) == 0,
                 "lamq_kl_head: the distribution's rows must be 16-byte aligned with ldp >= V");
    LAMQ_REQUIRE(workspace_bytes >= lamq_kl_workspace_size(ntok), "lamq_kl_head: workspace too small");
    cudaStream_t s = (cudaStream_t)stream;
    KLLayout l;
    float *pm, *ps;
    double *pbv, *sums;
    st = run_pass(kModeProbe, H, ldh, ntok, d, E, lde, V, const_cast<float *>(pdist), ldp, nullptr, workspace, status,
                  s, l, &pm, &ps, &pbv, &sums);
    if (st) return st;
    kl_combine_kernel<<<kCombineBlocks, 256, 0, s>>>(kModeProbe, ntok, kVSplit, pm, ps, pbv, nullptr,
                                                     const_cast<double *>(stat_a), const_cast<double *>(stat_p),
                                                     lse_ref, w, kl_pos, sums);
    LAMQ_CHECK_LAUNCH("lamq_kl_head combine");
    kl_total_kernel<<<1, 1, 0, s>>>(sums, kCombineBlocks, kl_out);
    LAMQ_CHECK_LAUNCH("lamq_kl_head total");
    return LAMQ_OK;
}
