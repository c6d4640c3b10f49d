// k_gemm_tc.cu -- batched Q8 weight-only GEMM on the 5th-generation tensor
// cores (tcgen05, TMEM accumulators, bulk-copy staging), dequantising in
// shared memory.
//
//   y[b, n] = s_n * sum_k x[b, k] * q[n, k]      (+ bias / alpha / beta epilogue)
//
// the batched form of AexisGemm2DPack4LinearTextureAFromLinear with INT8
// weights and per-output-row scales (HLSL Pack4Matmul:1038-1104, weight read
// AexisGemm2DReadB :707-734). The per-row scale is constant along K, so the
// tensor cores multiply the exact int8 values (as fp16) and the scale is
// applied once per output in the epilogue.
//
// Layout:
//   * weights, repacked once per handle: [N/128][K/64] blocks of 128 rows x 64
//     int8 (8 KB contiguous), so one k-block of a 128-row slab is one bulk copy;
//   * activations, prepared per call: [K/64][NB rows][64] fp16 in the 128-byte
//     swizzled K-major layout the MMA descriptors describe (8-row atoms of
//     1024 bytes). fp32 activations are split into fp16 hi and lo rows
//     (x = hi + lo to about 22 bits) that ride in the same MMA as extra
//     columns, so fp32 inputs keep fp32-class accuracy.
// Per CTA (persistent, one per SM): a contiguous range of 128-row slabs,
// taken two per accumulator tile (two M=128 MMAs sharing the activation tile)
// when two such tiles fit in TMEM (MMA width nb <= 128), else one, each over
// all K. TMEM holds two accumulator tiles: tile t accumulates into buffer
// t & 1 while the epilogue drains tile t - 1 from the other, so the output
// stores overlap the next tile's weight stream, dequantisation and MMAs.
// Three shared-memory rings decouple the latencies: int8 weights (up to 8
// k-blocks deep, freed as soon as they are dequantised), fp16 A tiles (2
// deep, freed by the MMA commit) and activations (3-4 deep, freed by the MMA
// commit). Warp roles: 0 int8 bulk-copy producer, 1 MMA issuer and TMEM
// owner, 2-5 dequantise int8 -> fp16 into the swizzled A tiles, 6 activation
// bulk-copy producer, 7-10 the epilogue (TMEM -> registers -> staging buffers
// of their own -> 16-byte row stores). Every barrier wait is bounded.
#include "gemv_dev.cuh"

namespace {

using namespace aexis_dev;

constexpr int kTcThreads = 352;          // 11 warps
constexpr int kTM = 128;                 // rows per MMA (M) = rows per slab
constexpr int kTile = 256;               // at most two slabs per accumulator tile
constexpr int kKB = 64;                  // K per stage (one 128-byte swizzle atom of fp16)
constexpr int kSlabBytes = kTM * kKB;    // int8 bytes of one slab k-block (8 KB)
constexpr int kATileBytes = kTM * 128;   // fp16 bytes of one slab k-block (16 KB)
constexpr int kADepth = 2;               // fp16 A ring
constexpr int kMaxDepth = 8;             // int8 and activation rings
constexpr int kSmemBudget = 227 * 1024;
constexpr int kStgBytes = 32 * kTM * 4;  // one epilogue staging buffer: 32 output rows x 128 outputs, fp32
constexpr int kStgBufs = 4;

// Slabs per accumulator tile: two when two such tiles (2 x 2 x nb columns)
// fit in the 512 TMEM columns, else one.
__host__ __device__ inline int tc_tile_slabs(int nb) { return 4 * nb <= 512 ? 2 : 1; }

struct TcParams {
    const uint8_t* wt;        // tiled int8 weights
    const void* scales;       // per row
    int scale_f16;
    const uint8_t* xt;        // prepared activations [K/64][nb][128 B]
    int n, k, m, nb, split;   // nb = MMA N (rows of xt), split: hi rows [0,m), lo rows [nb/2, nb/2+m)
    int n_slabs;              // ceil(n / 128)
    int raw_depth, b_depth;   // ring depths (int8 weights, activations)
    const float* bias;
    float alpha, beta;
    void* y;
    int y_f16, ldy;
    int tiled;                // 1: beta*bias + alpha*acc (lm_head form)
    int bulk_out;             // y and its row stride 16-byte aligned: staged row stores
    int k_splits;             // > 1: work units are (slab, K range), one slab per tile
    int accumulate;           // 1: y += result with fp32 atomics (bias from the first K range)
    int* status;
};

// Tile t of a CTA's work range [lo, hi): slabs [slab0, slab0 + ns) over
// k-blocks [kb0, kb1); `first` when the tile starts at k-block 0.
struct TcTile {
    int slab0, ns, kb0, kb1, first;
};

__device__ __forceinline__ TcTile tc_tile(const TcParams& p, int lo, int hi, int t, int nkb) {
    TcTile T;
    if (p.k_splits <= 1) {
        const int ts = tc_tile_slabs(p.nb);
        T.slab0 = lo + ts * t;
        T.ns = hi - T.slab0 < ts ? hi - T.slab0 : ts;
        T.kb0 = 0;
        T.kb1 = nkb;
    } else {
        const int u = lo + t, ks = u % p.k_splits;
        T.slab0 = u / p.k_splits;
        T.ns = 1;
        T.kb0 = ks * nkb / p.k_splits;
        T.kb1 = (ks + 1) * nkb / p.k_splits;
    }
    T.first = T.kb0 == 0;
    return T;
}

// Shared-memory carve-up (offsets from a 1024-aligned base): the fp16 A ring
// (kADepth x one tile's slabs), the activation ring, the epilogue staging
// buffers, the int8 ring (one tile's slabs per stage), the barriers.
struct TcLayout {
    int ts, b_bytes, b_stage, a_stage, raw_stage, a_off, b_off, stg_off, raw_off, bar_off, total;
};

__host__ __device__ inline TcLayout tc_layout(int nb, int raw_depth, int b_depth) {
    TcLayout L;
    L.ts = tc_tile_slabs(nb);
    L.b_bytes = nb * 128;
    L.b_stage = (L.b_bytes + 1023) & ~1023;
    L.a_stage = L.ts * kATileBytes;
    L.raw_stage = L.ts * kSlabBytes;
    L.a_off = 0;
    L.b_off = kADepth * L.a_stage;
    L.stg_off = L.b_off + b_depth * L.b_stage;
    L.raw_off = L.stg_off + kStgBufs * kStgBytes;
    L.bar_off = L.raw_off + raw_depth * L.raw_stage;
    L.total = L.bar_off + 512;
    return L;
}

// Ring depths for MMA width nb: activations 3 deep at nb >= 128, else 4; the
// int8 ring takes what is left, up to 8. False when fewer than 2 fit.
bool tc_depths(int nb, int& raw_depth, int& b_depth) {
    const int b_stage = (nb * 128 + 1023) & ~1023;
    const int ts = tc_tile_slabs(nb);
    b_depth = nb >= 128 ? 3 : 4;
    const int avail = kSmemBudget - 1024 - 512 - kADepth * ts * kATileBytes - b_depth * b_stage - kStgBufs * kStgBytes;
    raw_depth = avail / (ts * kSlabBytes);
    if (raw_depth > kMaxDepth) raw_depth = kMaxDepth;
    return raw_depth >= 2;
}

__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
    // K-major, 128-byte swizzle: 8-row atoms 1024 bytes apart (SBO), LBO 1,
    // version 1 (sm_100), layout type 2.
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;                      // LBO (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;            // SBO
    d |= (uint64_t)1 << 46;                      // version
    d |= (uint64_t)2 << 61;                      // SWIZZLE_128B
    return d;
}

__device__ __forceinline__ uint32_t idesc_f16_f32(int m, int n) {
    // c_format F32 (bit 4), a/b F16, both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, int accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 16 consecutive TMEM columns of this thread's lane; complete after tmem_wait().
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }


// int8 x4 (one word) -> two fp16x2 of the exact values: bytes biased by 128
// (XOR) and placed under the fp16 exponent of 1024 with PRMT, then 1024+128
// subtracted (exact in fp16).
__device__ __forceinline__ void i8x4_to_h2x2(uint32_t v, uint32_t& lo, uint32_t& hi) {
    const uint32_t u = v ^ 0x80808080u;
    uint32_t a = __byte_perm(u, 0x64646464u, 0x4140);
    uint32_t b = __byte_perm(u, 0x64646464u, 0x4342);
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
    __half2 ha = __hsub2(*reinterpret_cast<__half2*>(&a), bias);
    __half2 hb = __hsub2(*reinterpret_cast<__half2*>(&b), bias);
    lo = *reinterpret_cast<uint32_t*>(&ha);
    hi = *reinterpret_cast<uint32_t*>(&hb);
}

__global__ void __launch_bounds__(kTcThreads, 1) gemm_q8_tc_kernel(TcParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const TcLayout L = tc_layout(p.nb, p.raw_depth, p.b_depth);
    const int RD = p.raw_depth, BD = p.b_depth;
    uint64_t* bars = reinterpret_cast<uint64_t*>(base + L.bar_off);
    uint64_t* raw_full = bars;                    // int8 producer tx
    uint64_t* raw_empty = bars + kMaxDepth;       // 4 dequant warps
    uint64_t* b_full = bars + 2 * kMaxDepth;      // activation producer tx
    uint64_t* b_empty = bars + 3 * kMaxDepth;     // MMA commit
    uint64_t* a_ready = bars + 4 * kMaxDepth;     // 4 dequant warps
    uint64_t* a_empty = a_ready + kADepth;        // MMA commit
    uint64_t* acc_full = a_empty + kADepth;       // [2] MMA commit after a tile (per TMEM buffer)
    uint64_t* acc_empty = acc_full + 2;           // [2] 4 epilogue warps
    uint64_t* drain = acc_empty + 2;              // final MMA commit before TMEM is freed
    uint64_t* stg_full = drain + 1;               // 4 epilogue staging buffers: 128 writers
    uint64_t* stg_free = stg_full + 4;            // 128 readers done with the buffer
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(stg_free + 4);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nkb = p.k / kKB;
    // A contiguous range of work per CTA (counts differ by at most one):
    // 128-row slabs taken two per accumulator tile, or with k_splits > 1
    // (slab, K range) units taken one per tile.
    const int units = p.k_splits > 1 ? p.n_slabs * p.k_splits : p.n_slabs;
    const int s_lo = (int)((long long)blockIdx.x * units / gridDim.x);
    const int s_hi = (int)((long long)(blockIdx.x + 1) * units / gridDim.x);
    const int ts = L.ts;
    const int my_tiles = p.k_splits > 1 ? s_hi - s_lo : (s_hi - s_lo + ts - 1) / ts;
    // Two accumulator tiles of ts x nb columns each.
    const int acc_cols = ts * p.nb;
    const uint32_t tmem_cols = (uint32_t)(2 * acc_cols <= 32 ? 32 : (2 * acc_cols <= 64 ? 64 :
                                          (2 * acc_cols <= 128 ? 128 : (2 * acc_cols <= 256 ? 256 : 512))));

    if (threadIdx.x == 0) {
        for (int s = 0; s < kMaxDepth; ++s) {
            mbar_init(raw_full + s, 1);
            mbar_init(raw_empty + s, 4);
            mbar_init(b_full + s, 1);
            mbar_init(b_empty + s, 1);
        }
        for (int s = 0; s < kADepth; ++s) {
            mbar_init(a_ready + s, 4);
            mbar_init(a_empty + s, 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(acc_full + s, 1);
            mbar_init(acc_empty + s, 4);
        }
        mbar_init(drain, 1);
        for (int s = 0; s < 4; ++s) {
            mbar_init(stg_full + s, 128);
            mbar_init(stg_free + s, 128);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(tmem_slot)), "r"(tmem_cols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // Programmatic dependent launch: the weights are immutable, so their bulk
    // copies (warp 0) and dequantisation (warps 2-5) start before the wait on
    // the previous kernel; the activation producer (6), the MMA issuer (1)
    // and every epilogue wait first. The CTA lets its dependents launch only
    // after that wait (warps 1 and 6), so a dependent's own pre-wait reads
    // never see a kernel older than this one still running.

    if (warp == 0) {
        // ------------------------------------------------- int8 weight producer
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            int it = 0, issued = 0;
            for (int t = 0; t < my_tiles && !*abort_flag; ++t) {
                const TcTile T = tc_tile(p, s_lo, s_hi, t, nkb);
                const int slab0 = T.slab0, ns = T.ns;
                for (int kb = T.kb0; kb < T.kb1; ++kb, ++it) {
                    const int s = it % RD;
                    if (it >= RD && !mbar_wait(raw_empty + s, ((it / RD) & 1) ^ 1)) {
                        report_timeout(p.status);
                        *abort_flag = 1;
                        break;
                    }
                    if (*abort_flag) break;
                    uint8_t* st = base + L.raw_off + s * L.raw_stage;
                    mbar_arrive_expect_tx(raw_full + s, (uint32_t)(ns * kSlabBytes));
                    for (int j = 0; j < ns; ++j)
                        bulk_g2s(st + j * kSlabBytes, p.wt + ((size_t)(slab0 + j) * nkb + kb) * kSlabBytes,
                                 (uint32_t)kSlabBytes, raw_full + s, pol);
                    issued = it + 1;
                }
            }
            // No bulk copy may still be landing when the CTA exits (the
            // consumers wait for every stage on the normal path).
            for (int i = issued - RD < 0 ? 0 : issued - RD; i < issued; ++i)
                if (!mbar_wait(raw_full + i % RD, (i / RD) & 1)) { report_timeout(p.status); break; }
        }
    } else if (warp == 6) {
        // ---------------------------------------------- activation producer
        griddep_wait();
        griddep_launch();
        if (lane == 0) {
            int it = 0, issued = 0;
            for (int t = 0; t < my_tiles && !*abort_flag; ++t) {
                const TcTile T = tc_tile(p, s_lo, s_hi, t, nkb);
                for (int kb = T.kb0; kb < T.kb1; ++kb, ++it) {
                    const int s = it % BD;
                    if (it >= BD && !mbar_wait(b_empty + s, ((it / BD) & 1) ^ 1)) {
                        report_timeout(p.status);
                        *abort_flag = 1;
                        break;
                    }
                    if (*abort_flag) break;
                    mbar_arrive_expect_tx(b_full + s, (uint32_t)L.b_bytes);
                    bulk_g2s_plain(base + L.b_off + s * L.b_stage, p.xt + (size_t)kb * L.b_bytes,
                                   (uint32_t)L.b_bytes, b_full + s);
                    issued = it + 1;
                }
            }
            for (int i = issued - BD < 0 ? 0 : issued - BD; i < issued; ++i)
                if (!mbar_wait(b_full + i % BD, (i / BD) & 1)) { report_timeout(p.status); break; }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA issuer
        griddep_wait();
        griddep_launch();
        if (lane == 0) {
            // tcgen05.mma issue blocks this thread about as long as the MMA
            // runs, so the tensor pipe idles during whatever the thread does
            // between k-blocks: that bookkeeping is kept to increments.
            // Stage / phase counters advance by one; the smem descriptors of
            // stage 0 are built once and advanced by the stage stride and by
            // 32 bytes (2 units of the 16-byte start field) per K=16 step.
            const uint32_t idesc = idesc_f16_f32(kTM, p.nb);
            const uint64_t adesc0 = sw128_desc(smem_u32(base + L.a_off));
            const uint64_t bdesc0 = sw128_desc(smem_u32(base + L.b_off));
            const uint64_t a_step = (uint64_t)(L.a_stage >> 4), b_step = (uint64_t)(L.b_stage >> 4);
            const uint64_t slab_step = (uint64_t)(kATileBytes >> 4);
            int sa = 0, sb = 0;
            uint32_t pa = 0, pb = 0;
            uint64_t adesc = adesc0, bdesc = bdesc0;
            bool ok = true;
            for (int t = 0; t < my_tiles && ok; ++t) {
                const TcTile T = tc_tile(p, s_lo, s_hi, t, nkb);
                const int ns = T.ns;
                const uint32_t acc = tmem + (uint32_t)((t & 1) * acc_cols);
                // Buffer t & 1 was last drained by the epilogue of tile t - 2.
                if (t >= 2 && !mbar_wait(acc_empty + (t & 1), ((t >> 1) + 1) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int kb = T.kb0; kb < T.kb1; ++kb) {
                    if (!mbar_wait(a_ready + sa, pa) || !mbar_wait(b_full + sb, pb)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const int first = kb == T.kb0;
#pragma unroll
                    for (int kk = 0; kk < kKB / 16; ++kk)
                        mma_f16(acc, adesc + 2 * kk, bdesc + 2 * kk, idesc, (first && kk == 0) ? 0 : 1);
                    if (ns > 1) {
#pragma unroll
                        for (int kk = 0; kk < kKB / 16; ++kk)
                            mma_f16(acc + (uint32_t)p.nb, adesc + slab_step + 2 * kk, bdesc + 2 * kk, idesc,
                                    (first && kk == 0) ? 0 : 1);
                    }
                    mma_commit(a_empty + sa);
                    mma_commit(b_empty + sb);
                    if (++sa == kADepth) {
                        sa = 0;
                        pa ^= 1u;
                        adesc = adesc0;
                    } else {
                        adesc += a_step;
                    }
                    if (++sb == BD) {
                        sb = 0;
                        pb ^= 1u;
                        bdesc = bdesc0;
                    } else {
                        bdesc += b_step;
                    }
                }
                if (!ok || *abort_flag) {
                    ok = false;
                    break;
                }
                mma_commit(acc_full + (t & 1));
            }
            if (!ok) {
                report_timeout(p.status);
                *abort_flag = 1;
            }
            // Every MMA this thread issued has completed before TMEM is freed.
            mma_commit(drain);
            if (!mbar_wait(drain, 0)) report_timeout(p.status);
        }
    } else if (warp >= 2 && warp <= 5) {
        // ------------------------------------------ dequantise int8 -> fp16 (2..5)
        const int dw = warp - 2;              // 0..3
        const int dt = dw * 32 + lane;        // 0..127
        int it = 0;
        for (int t = 0; t < my_tiles && !*abort_flag; ++t) {
            const TcTile T = tc_tile(p, s_lo, s_hi, t, nkb);
            const int ns = T.ns;
            for (int kb = T.kb0; kb < T.kb1; ++kb, ++it) {
                const int sr = it % RD, sa = it % kADepth;
                if (!mbar_wait(raw_full + sr, (it / RD) & 1) ||
                    (it >= kADepth && !mbar_wait(a_empty + sa, ((it / kADepth) & 1) ^ 1))) {
                    report_timeout(p.status);
                    *abort_flag = 1;
                    break;
                }
                const uint8_t* st = base + L.raw_off + sr * L.raw_stage;
                uint8_t* a_t = base + L.a_off + sa * L.a_stage;
                // Thread dt converts 16 int8 (chunk dt & 3 of row dt >> 2) of
                // each 32-row group: conflict-free reads and swizzled writes.
#pragma unroll 2
                for (int g = 0; g < ns * (kTM / 32); ++g) {
                    const int row = g * 32 + (dt >> 2);          // 0..255
                    const int ch = dt & 3;                       // 16-byte chunk of the 64 int8
                    const uint4 q = *reinterpret_cast<const uint4*>(st + row * kKB + ch * 16);
                    uint32_t h[8];
                    i8x4_to_h2x2(q.x, h[0], h[1]);
                    i8x4_to_h2x2(q.y, h[2], h[3]);
                    i8x4_to_h2x2(q.z, h[4], h[5]);
                    i8x4_to_h2x2(q.w, h[6], h[7]);
                    const int j = row >> 7, r = row & 127;
                    uint8_t* arow = a_t + j * kTM * 128 + (r >> 3) * 1024 + (r & 7) * 128;
                    const int c0 = 2 * ch, c1 = 2 * ch + 1;     // fp16 16-byte chunks
                    *reinterpret_cast<uint4*>(arow + ((c0 ^ (r & 7)) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
                    *reinterpret_cast<uint4*>(arow + ((c1 ^ (r & 7)) << 4)) = make_uint4(h[4], h[5], h[6], h[7]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(raw_empty + sr);
                    mbar_arrive(a_ready + sa);
                }
            }
        }
    } else {
        // ------------------------------------------------------ epilogue (7..10)
        const int dw = warp - 7;              // 0..3: output rows dw, dw + 4, ... of a staged chunk
        const int quad = warp & 3;            // TMEM lane quadrant this warp may access
        int chunk = 0;                        // staged epilogue chunks so far (all tiles)
        for (int t = 0; t < my_tiles && !*abort_flag; ++t) {
            const TcTile T = tc_tile(p, s_lo, s_hi, t, nkb);
            const int slab0 = T.slab0, ns = T.ns;
            // Wait for the tile's accumulators (TMEM buffer t & 1), then each thread owns
            // one weight row (TMEM lane) of each 128-row slab. The outputs and
            // the bias belong to the stream order: after the previous kernel.
            griddep_wait();
            if (!mbar_wait(acc_full + (t & 1), (t >> 1) & 1)) {
                report_timeout(p.status);
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            // Column b < m of the accumulator is output row b; with split
            // activations its lo part sits in column hi_cols + b, so both
            // halves of a chunk load side by side and nothing is re-read.
            const int mrows = p.m;
            const int hi_cols = p.split ? p.nb >> 1 : p.nb;
            const size_t ldy = (size_t)p.ldy;
            const int esz = p.y_f16 ? 2 : 4;
            for (int j = 0; j < ns; ++j) {
                const int slab = slab0 + j;
                const int n = slab * kTM + quad * 32 + lane;
                const bool nvalid = n < p.n;
                float sc = 0.0f, bb = 0.0f;
                if (nvalid) {
                    sc = p.scale_f16 ? __half2float(reinterpret_cast<const __half*>(p.scales)[n])
                                     : reinterpret_cast<const float*>(p.scales)[n];
                    bb = p.bias && T.first ? p.beta * p.bias[n] : 0.0f;
                }
                const uint32_t lane_addr =
                    tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)((t & 1) * acc_cols + j * p.nb);
                const int cnt = p.n - slab * kTM < kTM ? p.n - slab * kTM : kTM;  // valid outputs of the slab
                if (p.bulk_out && ((cnt * esz) & 15) == 0) {
                    // Staged path: 32 output rows at a time are transposed
                    // through shared memory (four 16 KB buffers of the
                    // epilogue's own, rotating), then each warp writes whole
                    // 128-output row segments with 16-byte (8-byte for fp16)
                    // stores: a quarter of the store instructions of the
                    // lane-per-output layout TMEM delivers.
                    for (int c0 = 0; c0 < mrows && !*abort_flag; c0 += 32, ++chunk) {
                        const int nrows = mrows - c0 < 32 ? mrows - c0 : 32;
                        const int buf = chunk & 3;
                        const uint32_t use = (uint32_t)(chunk >> 2);
                        if (chunk >= 4 && !mbar_wait(stg_free + buf, (use - 1) & 1)) {
                            report_timeout(p.status);
                            *abort_flag = 1;
                            break;
                        }
                        uint32_t r[32], q[32];
                        tmem_ld16(lane_addr + (uint32_t)c0, r);
                        if (nrows > 16) tmem_ld16(lane_addr + (uint32_t)(c0 + 16), r + 16);
                        if (p.split) {
                            tmem_ld16(lane_addr + (uint32_t)(hi_cols + c0), q);
                            if (nrows > 16) tmem_ld16(lane_addr + (uint32_t)(hi_cols + c0 + 16), q + 16);
                        }
                        tmem_wait();
                        float* stg = reinterpret_cast<float*>(base + L.stg_off + buf * kStgBytes);
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            float acc = __uint_as_float(r[i]);
                            if (p.split) acc += __uint_as_float(q[i]);
                            const float out = p.tiled ? bb + p.alpha * (acc * sc) : p.alpha * (bb + acc * sc);
                            if (i < nrows) stg[i * kTM + quad * 32 + lane] = out;
                        }
                        mbar_arrive(stg_full + buf);
                        if (!mbar_wait(stg_full + buf, use & 1)) {
                            report_timeout(p.status);
                            *abort_flag = 1;
                            break;
                        }
                        // Warp dw writes rows dw, dw + 4, ...: lane covers outputs 4 lane .. 4 lane + 3.
                        for (int i = dw; i < nrows; i += 4) {
                            const float4 v = *reinterpret_cast<const float4*>(stg + i * kTM + lane * 4);
                            if (lane * 4 < cnt) {
                                const size_t off = (size_t)(c0 + i) * ldy + (size_t)slab * kTM + lane * 4;
                                if (p.y_f16) {
                                    const __half2 h0 = __floats2half2_rn(v.x, v.y), h1 = __floats2half2_rn(v.z, v.w);
                                    uint2 u;
                                    u.x = *reinterpret_cast<const uint32_t*>(&h0);
                                    u.y = *reinterpret_cast<const uint32_t*>(&h1);
                                    *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(p.y) + off) = u;
                                } else {
                                    float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.y) + off);
                                    if (p.accumulate) atomicAdd(dst, v);
                                    else *dst = v;
                                }
                            }
                        }
                        mbar_arrive(stg_free + buf);
                    }
                    continue;
                }
                float* yf = reinterpret_cast<float*>(p.y) + n;
                __half* yh = reinterpret_cast<__half*>(p.y) + n;
                for (int c0 = 0; c0 < mrows; c0 += 16) {
                    uint32_t r[16], q[16];
                    tmem_ld16(lane_addr + (uint32_t)c0, r);
                    if (p.split) tmem_ld16(lane_addr + (uint32_t)(hi_cols + c0), q);
                    tmem_wait();
                    if (!nvalid) continue;
                    const int lim = mrows - c0;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        float acc = __uint_as_float(r[i]);
                        if (p.split) acc += __uint_as_float(q[i]);
                        const float out = p.tiled ? bb + p.alpha * (acc * sc) : p.alpha * (bb + acc * sc);
                        if (i < lim) {
                            if (p.y_f16) yh[(size_t)(c0 + i) * ldy] = __float2half_rn(out);
                            else if (p.accumulate) atomicAdd(yf + (size_t)(c0 + i) * ldy, out);
                            else yf[(size_t)(c0 + i) * ldy] = out;
                        }
                    }
                }
            }
            // Every TMEM load of this tile has completed (tmem_wait): the MMA
            // warp may reuse the buffer for tile t + 2.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + (t & 1));
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols) : "memory");
    }
}

// Activations -> xt [K/64][nb][64] fp16, 128-byte swizzled rows, one CTA per
// output row b < nb/(split ? 2 : 1): hi = fp16(v) in row b and, with split,
// lo = fp16(v - hi) in row nb/2 + b; rows b >= m are zero. The value v is
//   op 0: x[b][k] (fp16 or fp32);
//   op 1: RMSNorm, x[b][k] * rsqrt(max(mean(x[b]^2) + eps, 1e-20)) * gamma[k]
//         (AexisRmsNormPack4LinearMat, AexisCommon.compute:4531-4563; x fp32);
//   op 2: SwiGLU of interleaved pairs, silu(x[b][2k]) * x[b][2k+1]
//         (HLSL Pack4Matmul:91-94, 118-128; x fp32).
// With `zero`, the CTA of row b also clears zero[b][0, zero_n) (the output
// of a following accumulating GEMM). Waits for the previous grid (PDL) and
// then lets its dependents launch, so a following GEMM streams its weights
// during this kernel.
__global__ void __launch_bounds__(256) tc_prep_kernel(const void* x, int x_f16, int lda, int m, int k, int op,
                                                      const float* gamma, float eps, int nb, int split, uint8_t* xt,
                                                      float* zero, int zero_ld, int zero_n) {
    __shared__ float red[8];
    griddep_wait();
    griddep_launch();  // after the wait: a dependent's pre-wait reads see every older kernel complete
    const int b = blockIdx.x;
    const int half = split ? nb >> 1 : nb;
    const float* xf = reinterpret_cast<const float*>(x);
    const long long row = (long long)b * lda;
    float inv = 1.0f;
    if (op == 1 && b < m) {
        float ss = 0.0f;
        for (int i = threadIdx.x; i < k; i += 256) ss = fmaf(xf[row + i], xf[row + i], ss);
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();
        float tot = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) tot += red[w];
        inv = 1.0f / sqrtf(fmaxf(tot / (float)k + eps, 1e-20f));
    }
    for (int c8 = threadIdx.x; c8 < k / 8; c8 += 256) {
        __half hi[8], lo[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int kk = c8 * 8 + e;
            float v = 0.0f;
            if (b < m) {
                if (op == 0) {
                    v = aexis_load_act(x, x_f16 ? AEXIS_F16 : AEXIS_F32, row + kk);
                } else if (op == 1) {
                    v = xf[row + kk] * inv * gamma[kk];
                } else {
                    const float g = xf[row + 2 * kk], u = xf[row + 2 * kk + 1];
                    v = __fmul_rn(g / (1.0f + expf(-g)), u);
                }
            }
            hi[e] = __float2half_rn(v);
            lo[e] = __float2half_rn(v - __half2float(hi[e]));
        }
        const int kb = c8 >> 3, c = c8 & 7;
        *reinterpret_cast<uint4*>(xt + ((size_t)kb * nb + b) * 128 + ((c ^ (b & 7)) << 4)) =
            *reinterpret_cast<const uint4*>(hi);
        if (split) {
            const int r = half + b;
            *reinterpret_cast<uint4*>(xt + ((size_t)kb * nb + r) * 128 + ((c ^ (r & 7)) << 4)) =
                *reinterpret_cast<const uint4*>(lo);
        }
    }
    if (zero && b < m)
        for (int i = threadIdx.x; i < zero_n; i += 256) zero[(long long)b * zero_ld + i] = 0.0f;
}

// Row-major Q8 [n][k] -> [ceil(n/256)*2][k/64][128][64] (rows past n zero;
// the slab count is even so a 256-row CTA tile never reads past the buffer).
__global__ void repack_q8_kernel(const uint8_t* src, int n, int k, uint8_t* dst) {
    const int nkb = k / kKB;
    const long long total = (long long)((n + kTile - 1) / kTile) * kTile * nkb * 4;  // 16-byte chunks
    for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (long long)gridDim.x * blockDim.x) {
        const int ch = (int)(t & 3);
        const long long rowblk = t >> 2;                 // (slab, kb, r)
        const int r = (int)(rowblk % kTM);
        const long long sk = rowblk / kTM;
        const int kb = (int)(sk % nkb);
        const long long slab = sk / nkb;
        const long long row = slab * kTM + r;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (row < n) v = *reinterpret_cast<const uint4*>(src + row * k + kb * kKB + ch * 16);
        *reinterpret_cast<uint4*>(dst + ((slab * nkb + kb) * kTM + r) * kKB + ch * 16) = v;
    }
}

}  // namespace

// MMA width (rows of the prepared activations): m rounded up to 16, twice
// that for split fp32 activations.
int tc_width(int m, int a_dtype) {
    const int mp = (m + 15) / 16 * 16;
    return a_dtype == AEXIS_F32 ? 2 * mp : mp;
}

size_t gemm_tc_smem_bytes(int nb) {
    int rd = 0, bd = 0;
    if (!tc_depths(nb, rd, bd)) return (size_t)1 << 30;
    return 1024 + (size_t)tc_layout(nb, rd, bd).total;  // + alignment slack
}

bool gemm_tc_supported(const aexis_weights* w, int m, int a_dtype) {
    if (w->kind != WK_Q8 || w->k % kKB != 0 || m < 1) return false;
    const int nb = tc_width(m, a_dtype);
    return nb <= 256 && gemm_tc_smem_bytes(nb) <= (size_t)kSmemBudget;
}

size_t gemm_tc_tiled_bytes(const aexis_weights* w) {
    return (size_t)((w->n + kTile - 1) / kTile) * kTile * w->k;
}

cudaError_t launch_repack_q8(const aexis_weights* w, void* tiled, cudaStream_t s) {
    repack_q8_kernel<<<148 * 8, 256, 0, s>>>(reinterpret_cast<const uint8_t*>(w->data), w->n, w->k,
                                              reinterpret_cast<uint8_t*>(tiled));
    return cudaGetLastError();
}

size_t gemm_tc_xt_bytes(int m, int k, int a_dtype) {
    return (size_t)k * tc_width(m, a_dtype) * 2;
}

namespace {

cudaError_t launch_maybe_pdl(const void* fn, dim3 grid, dim3 block, size_t smem, bool pdl, cudaStream_t s,
                             void** args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace

cudaError_t launch_tc_prep(int op, const void* x, int x_f16, int lda, int m, int k, const float* gamma, float eps,
                           int split, void* xt, float* zero, int zero_ld, int zero_n, bool pdl, cudaStream_t s) {
    const int nb = tc_width(m, split ? AEXIS_F32 : AEXIS_F16);
    const int rows = split ? nb / 2 : nb;
    uint8_t* xtp = reinterpret_cast<uint8_t*>(xt);
    void* args[] = {(void*)&x, &x_f16, &lda, &m, &k, &op, (void*)&gamma, &eps, (void*)&nb, &split, &xtp,
                    &zero, &zero_ld, &zero_n};
    return launch_maybe_pdl((const void*)tc_prep_kernel, dim3(rows), dim3(256), 0, pdl, s, args);
}

cudaError_t launch_gemm_tc_prepared(const TcLaunch& a, cudaStream_t s) {
    const aexis_weights* w = a.w;
    const int nb = tc_width(a.m, a.split ? AEXIS_F32 : AEXIS_F16);
    if (a.accumulate && a.y_dtype != AEXIS_F32) return cudaErrorNotSupported;
    TcParams p = {};
    p.wt = reinterpret_cast<const uint8_t*>(a.tiled);
    p.scales = w->scales;
    p.scale_f16 = w->scale_dtype == AEXIS_F16;
    p.xt = reinterpret_cast<const uint8_t*>(a.xt);
    p.n = w->n;
    p.k = w->k;
    p.m = a.m;
    p.nb = nb;
    p.split = a.split;
    p.n_slabs = (w->n + kTM - 1) / kTM;
    if (!tc_depths(nb, p.raw_depth, p.b_depth)) return cudaErrorNotSupported;
    p.bias = a.bias;
    p.alpha = a.alpha;
    p.beta = a.beta;
    p.y = a.y;
    p.y_f16 = a.y_dtype == AEXIS_F16;
    p.ldy = a.ldy;
    p.tiled = a.tiled_epi;
    const int esz = p.y_f16 ? 2 : 4;
    p.bulk_out = (reinterpret_cast<uintptr_t>(a.y) & 15) == 0 && (((size_t)a.ldy * esz) & 15) == 0;
    p.accumulate = a.accumulate;
    // Split K only when accumulating and the slabs alone would leave SMs idle.
    // The automatic split aims at about two thirds of the SMs (rounded up per
    // slab) and keeps at least two k-blocks per K range: a range's fixed cost
    // (prologue, epilogue, atomics) outweighs a k-block's work. Config 4:
    // 1.525 ms per step with one range per SM, 1.498 with the two-block cap,
    // 1.425 with both.
    const int nkb = w->k / kKB;
    int ks = 1;
    if (a.accumulate && p.n_slabs < a.sm_count) {
        const int cap = a.k_splits > 0 ? nkb : (nkb / 2 > 1 ? nkb / 2 : 1);
        ks = a.k_splits > 0 ? a.k_splits : (a.sm_count * 2 / 3 + p.n_slabs - 1) / p.n_slabs;
        ks = ks > cap ? cap : (ks < 1 ? 1 : ks);
    }
    p.k_splits = ks;
    p.status = a.status;
    const size_t smem = gemm_tc_smem_bytes(nb);
    int dev = 0;
    cudaGetDevice(&dev);
    static size_t configured[64] = {};
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (smem > configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemm_q8_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured[dev] = smem;
    }
    const int units = ks > 1 ? p.n_slabs * ks : p.n_slabs;
    const int grid = units < a.sm_count ? units : a.sm_count;
    void* args[] = {&p};
    return launch_maybe_pdl((const void*)gemm_q8_tc_kernel, dim3(grid), dim3(kTcThreads), smem, a.pdl, s, args);
}

cudaError_t launch_gemm_tc(const aexis_weights* w, const void* tiled, const void* x, int a_dtype, int lda, int m,
                           void* xt, const float* bias, float alpha, float beta, void* y, int y_dtype, int ldy,
                           int tiled_epi, int sm_count, int* status, cudaStream_t s) {
    const int split = a_dtype == AEXIS_F32;
    cudaError_t e = launch_tc_prep(0, x, a_dtype == AEXIS_F16, lda, m, w->k, nullptr, 0.0f, split, xt, nullptr, 0, 0,
                                   false, s);
    if (e != cudaSuccess) return e;
    TcLaunch a;
    a.w = w;
    a.tiled = tiled;
    a.xt = xt;
    a.m = m;
    a.split = split;
    a.bias = bias;
    a.alpha = alpha;
    a.beta = beta;
    a.y = y;
    a.y_dtype = y_dtype;
    a.ldy = ldy;
    a.tiled_epi = tiled_epi;
    a.sm_count = sm_count;
    a.status = status;
    return launch_gemm_tc_prepared(a, s);
}
