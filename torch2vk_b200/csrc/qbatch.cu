// Quantized linear for small token batches (5 .. 16 tokens per launch: decode
// at batch 5..16, the config-2 sweep's M = 16 points):
// y[m, n] = sum_k x[m, k] * deq(W)[n, k] over Q4_K rows, with the arithmetic
// of the decode matvecs (qlinear.cu) and of the reference's matvec shader
// (src/models/quantized_qwen3/shaders/linear_nobias_q4_k_matvec_f32.py:107-197):
// the fp16 x (with a fused RMSNorm: the normalized values rounded to fp16
// once) times the decoded weights in fp32, here on fp16 tensor cores.
//
// B200 design (weight streaming sets the pace):
//  * One 8-warp CTA per SM, thread-block clusters of C CTAs along K: CTA c of
//    a cluster owns K slice c (K / C values) and keeps its x slice for all
//    tokens in shared memory, so each weight byte is read once and meets
//    every token there.
//  * Each warp streams its own 32-row tile (two mma row tiles) through a ring
//    of 2-D TMA boxes (2 x 16 rows x 144 bytes = one Q4_K super-block of 32
//    rows per stage, bounded mbarrier waits, first stages requested before
//    griddepcontrol.wait).
//  * mma.sync m16n8k16 (f16 in, f32 accumulators): A = the nibbles as fp16
//    subnormals (q * 2^-24) times their sub-block scale code in one f16x2
//    multiply, exact (sc * q < 1024), so one accumulator holds a super-block;
//    B columns = tokens, so one A fragment serves up to two 8-token mma; the
//    min term sum_j m_j * xsum_j is one more mma per tile and token group
//    (B = the hi / lo fp16 parts of the sub-block sums).  d and dmin are
//    applied in fp32.
//  * The C partial tiles of a unit (8 tiles = 256 rows) meet through
//    distributed shared memory: warp w sends its tile to CTA w % C, which adds
//    the C partials in rank order (deterministic) and runs the epilogue
//    (+ residual, or SwiGLU of the gate and up halves of a tile).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdio.h>

#include "common.cuh"
#include "qgemm.cuh"

namespace t2c {
namespace {

constexpr int kBWarps = 8;
constexpr int kBThreads = kBWarps * 32;
constexpr int kBRows = 32;                 // rows per warp tile
constexpr int kBStage = kBRows * 144;      // one super-block of a tile
constexpr int kBMaxStages = 6;
constexpr int kBMaxC = 8;                  // cluster size along K
constexpr int kBMaxTokens = 16;
constexpr size_t kBSmemLimit = 227 * 1024;

struct BParams {
    alignas(64) CUtensorMap tmap[3];  // ROWS: the streams; SWIGLU: gate, up
    const __half *x;                  // [M, K]
    const float *norm_w;              // fp32 [K] or nullptr
    float eps;
    __half *y[3];
    const __half *res[3];
    int64_t n[3];           // rows per stream (SWIGLU: outputs)
    int64_t tile_begin[4];  // first tile of each stream; tile_begin[nstreams] = tiles
    int nstreams;
    int swiglu;
    int M;         // tokens in this launch
    int K;
    int C;         // cluster size (CTAs along K)
    int kc;        // K values per CTA
    int units;     // ceil(tiles / 8)
    int stages;
    int xrow;      // bytes per token of the x slice
    size_t off_x, off_stage;
};

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cl_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cl_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
__device__ __forceinline__ void st_cluster_f32(const void *local, uint32_t rank, float v) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

__device__ __forceinline__ void st_cluster_v4(const void *local, uint32_t rank, float a, float b, float c, float d) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(remote), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}

__device__ __forceinline__ uint4 lds128b(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds32b(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ void mma16816(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(__half lo, __half hi) {
    return static_cast<uint32_t>(__half_as_ushort(lo)) | (static_cast<uint32_t>(__half_as_ushort(hi)) << 16);
}
__device__ __forceinline__ uint32_t half2_dup_bits(float v) {
    const uint32_t b = __half_as_ushort(__float2half_rn(v));
    return b | (b << 16);
}

// x slice layout: per token, the kc values in pair-interleaved 4-value chunks
// (x0, x2, x1, x3) with 16 bytes of padding after every 16 chunks (row stride
// xrow, = 64 mod 128 so that the two tokens of a shared-memory phase fall in
// different banks), then per token and super-block the 8 sub-block sums as
// fp16 (hi[8], lo[8]).
__host__ __device__ __forceinline__ int bx_chunk_off(int c) { return 8 * c + 16 * (c >> 4); }
__host__ __device__ __forceinline__ int bx_row_bytes(int kc) {
    const int b = 2 * kc + (kc >> 6) * 16;
    return (b % 128 == 64) ? b : b + 64;
}

// Stages x (tokens [0, M), zeros up to T) of this CTA's slice, normalized when
// norm_w is given (the sum of squares of the whole row comes from all CTAs of
// the cluster through distributed shared memory).
template <int T>
__device__ void bx_prepare(const BParams &p, uint32_t crank, uint8_t *xs, uint8_t *xsum, float *sq, float *red) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int kc = p.kc, k0 = static_cast<int>(crank) * kc;
    const int cpr = kc >> 3;  // 8-value chunks per token row
    const int total = T * cpr;
    const int nsb = kc >> 8;
    float inv[T];
#pragma unroll
    for (int m = 0; m < T; ++m) inv[m] = 1.0f;
    if (p.norm_w != nullptr) {
        // this slice's sum of squares per token, then to every CTA of the cluster
        for (int m = warp; m < p.M; m += kBWarps) {
            float s = 0.0f;
            for (int c = lane; c < cpr; c += 32) {
                const uint4 v = *reinterpret_cast<const uint4 *>(p.x + static_cast<int64_t>(m) * p.K + k0 + 8 * c);
                const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 f = __half22float2(h[i]);
                    s = fmaf(f.x, f.x, fmaf(f.y, f.y, s));
                }
            }
            s = warp_sum(s);
            if (lane < p.C) st_cluster_f32(&sq[crank * kBMaxTokens + m], static_cast<uint32_t>(lane), s);
        }
        cl_arrive();
        cl_wait();
#pragma unroll
        for (int m = 0; m < T; ++m) {
            if (m < p.M) {
                float tot = 0.0f;
                for (int r = 0; r < p.C; ++r) tot += sq[r * kBMaxTokens + m];
                inv[m] = rsqrtf(tot / static_cast<float>(p.K) + p.eps);
            }
        }
    }
    (void)red;
    // lanes 4i .. 4i + 3 hold the four 8-value chunks of one 32-value sub-block
    for (int base = 0; base < total; base += kBThreads) {
        const int c = base + tid;
        const int m = c / cpr;
        const int v = (c - m * cpr) * 8;
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = 0.0f;
        if (c < total && m < p.M) {
            const uint4 raw = *reinterpret_cast<const uint4 *>(p.x + static_cast<int64_t>(m) * p.K + k0 + v);
            const __half2 *h = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 t2 = __half22float2(h[i]);
                f[2 * i] = t2.x;
                f[2 * i + 1] = t2.y;
            }
            if (p.norm_w != nullptr) {
                float r = 1.0f;
#pragma unroll
                for (int mm = 0; mm < T; ++mm)
                    if (mm == m) r = inv[mm];
                const float4 w0 = *reinterpret_cast<const float4 *>(p.norm_w + k0 + v);
                const float4 w1 = *reinterpret_cast<const float4 *>(p.norm_w + k0 + v + 4);
                const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = f[e] * r * wv[e];
            }
        }
        __half h[8];
        float sum = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            h[e] = __float2half_rn(f[e]);
            sum += __half2float(h[e]);
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if (c < total) {
            *reinterpret_cast<uint4 *>(xs + m * p.xrow + bx_chunk_off(v >> 2)) =
                make_uint4(pack_h2(h[0], h[2]), pack_h2(h[1], h[3]), pack_h2(h[4], h[6]), pack_h2(h[5], h[7]));
            if ((lane & 3) == 0) {
                const int j = v >> 5;
                const __half hi = __float2half_rn(sum);
                const __half lo = __float2half_rn(sum - __half2float(hi));
                uint8_t *dst = xsum + (m * nsb + (j >> 3)) * 32 + 2 * (j & 7);
                st_u16(dst, __half_as_ushort(hi));
                st_u16(dst + 16, __half_as_ushort(lo));
            }
        }
    }
    __syncthreads();
}

// Integer codes of sub-blocks 2t, 2t + 1 of a Q4_K header.
__device__ __forceinline__ void bq4k_codes(const uint4 h, int t, uint32_t &sc0, uint32_t &sc1, uint32_t &m0,
                                           uint32_t &m1) {
    const int i0 = (2 * t) & 3;
    const bool low = t < 2;
    const uint32_t y = h.y >> (8 * i0), z = h.z >> (8 * i0), w = h.w >> (8 * i0);
    const uint32_t scp = low ? (y & 0x3F3Fu) : ((w & 0x0F0Fu) | ((y >> 2) & 0x3030u));
    const uint32_t mnp = low ? (z & 0x3F3Fu) : (((w >> 4) & 0x0F0Fu) | ((z >> 2) & 0x3030u));
    sc0 = scp & 0xffu;
    sc1 = scp >> 8;
    m0 = mnp & 0xffu;
    m1 = mnp >> 8;
}

// Tile of unit u for warp w: stream, first row, whether it exists.
struct BTile {
    int si;
    int64_t row0;
    bool valid;
};

__device__ __forceinline__ BTile b_tile(const BParams &p, int64_t tile) {
    BTile r;
    r.valid = tile < p.tile_begin[p.nstreams];
    r.si = 0;
    if (p.swiglu) {
        r.row0 = tile * 16;
        return r;
    }
#pragma unroll
    for (int i = 1; i < 3; ++i)
        if (i < p.nstreams && tile >= p.tile_begin[i]) r.si = i;
    r.row0 = (tile - p.tile_begin[r.si]) * kBRows;
    return r;
}

// Requests item (tile, super-block sb) into a stage: two boxes of 16 rows x 144 bytes
// (ROWS: rows row0 .. row0 + 31 of the stream; SWIGLU: rows row0 .. row0 + 15 of gate, then of up).
__device__ __forceinline__ void b_issue(const BParams &p, const BTile &tl, int sb, uint8_t *stage, uint64_t *bar) {
    mbar_arrive_expect_tx(bar, static_cast<uint32_t>(kBStage));
    const int x = sb * 36;
    if (p.swiglu) {
        tma_load_2d(stage, &p.tmap[0], x, static_cast<int>(tl.row0), bar);
        tma_load_2d(stage + 16 * 144, &p.tmap[1], x, static_cast<int>(tl.row0), bar);
    } else {
        tma_load_2d(stage, &p.tmap[tl.si], x, static_cast<int>(tl.row0), bar);
        tma_load_2d(stage + 16 * 144, &p.tmap[tl.si], x, static_cast<int>(tl.row0) + 16, bar);
    }
}

// One super-block (local index j of the slice) of this warp's 32-row tile for all tokens.
template <int TG>
__device__ __forceinline__ void b_block(uint32_t stage, uint32_t xs, uint32_t xsum, int xrow, int nsb, int j,
                                        int lane, float acc[2][TG][4]) {
    const int g = lane >> 2, t = lane & 3;
    uint32_t W[2][2][8], scl[2][2], sch[2][2], mm[2][2];
    float d24[2][2], dmin[2][2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const uint32_t row = stage + static_cast<uint32_t>((16 * h + g + 8 * r) * 144);
            const uint4 hd = lds128b(row);
            const uint4 q0 = lds128b(row + 16 + 32 * t), q1 = lds128b(row + 32 + 32 * t);
            W[h][r][0] = q0.x;
            W[h][r][1] = q0.y;
            W[h][r][2] = q0.z;
            W[h][r][3] = q0.w;
            W[h][r][4] = q1.x;
            W[h][r][5] = q1.y;
            W[h][r][6] = q1.z;
            W[h][r][7] = q1.w;
            uint32_t c0, c1, n0, n1;
            bq4k_codes(hd, t, c0, c1, n0, n1);
            scl[h][r] = half2_dup_bits(static_cast<float>(c0));
            sch[h][r] = half2_dup_bits(static_cast<float>(c1) * 0.0625f);
            mm[h][r] = pack_h2(__float2half_rn(static_cast<float>(n0)), __float2half_rn(static_cast<float>(n1)));
            d24[h][r] = half_bits_to_float(hd.x) * 16777216.0f;
            dmin[h][r] = half_bits_to_float(hd.x >> 16);
        }
    }
    float D[2][TG][4];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int q = 0; q < TG; ++q)
#pragma unroll
            for (int i = 0; i < 4; ++i) D[h][q][i] = 0.0f;
    // B of token 8q + g: low / high chunks of group t of super-block j
    const uint32_t xb = xs + static_cast<uint32_t>(g * xrow + 576 * j + 144 * t);
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
        uint4 bl[TG], bh[TG];
#pragma unroll
        for (int q = 0; q < TG; ++q) {
            const uint32_t a = xb + static_cast<uint32_t>(8 * q * xrow + 16 * jj);
            bl[q] = lds128b(a);
            bh[q] = lds128b(a + 64);
        }
#pragma unroll
        for (int w2 = 0; w2 < 2; ++w2) {
            const int wj = 2 * jj + w2;
#pragma unroll
            for (int pp = 0; pp < 2; ++pp) {
                uint32_t a[2][4];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t w = pp ? (W[h][0][wj] >> 8) : W[h][0][wj];
                    const uint32_t v = pp ? (W[h][1][wj] >> 8) : W[h][1][wj];
                    a[h][0] = hmul2(w & 0x000F000Fu, scl[h][0]);
                    a[h][1] = hmul2(v & 0x000F000Fu, scl[h][1]);
                    a[h][2] = hmul2(w & 0x00F000F0u, sch[h][0]);
                    a[h][3] = hmul2(v & 0x00F000F0u, sch[h][1]);
                }
                const int c = 2 * w2 + pp;
#pragma unroll
                for (int q = 0; q < TG; ++q) {
                    const uint32_t b0 = c == 0 ? bl[q].x : c == 1 ? bl[q].y : c == 2 ? bl[q].z : bl[q].w;
                    const uint32_t b1 = c == 0 ? bh[q].x : c == 1 ? bh[q].y : c == 2 ? bh[q].z : bh[q].w;
#pragma unroll
                    for (int h = 0; h < 2; ++h) mma16816(D[h][q], a[h], b0, b1);
                }
            }
        }
    }
    // min term: sum_j m_j * xsum_j, then acc += d * D - dmin * E
#pragma unroll
    for (int q = 0; q < TG; ++q) {
        const uint32_t sa = xsum + static_cast<uint32_t>(((8 * q + g) * nsb + j) * 32 + 4 * t);
        const uint32_t e0 = lds32b(sa), e1 = lds32b(sa + 16);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float E[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            const uint32_t am[4] = {mm[h][0], mm[h][1], mm[h][0], mm[h][1]};
            mma16816(E, am, e0, e1);
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[h][q][i] += fmaf(d24[h][i >> 1], D[h][q][i], -dmin[h][i >> 1] * E[i]);
        }
    }
}

__device__ __forceinline__ float silu_b(float g) { return g / (1.0f + __expf(-g)); }

template <int TG>
__global__ void __launch_bounds__(kBThreads, 1) qbatch_kernel(const __grid_constant__ BParams p) {
    constexpr int T = 8 * TG;
    // a partial tile in the receive buffer: [part = h * TG + q][lane][4 floats] (lane (g, t), element i:
    // row 16 h + g + 8 (i >> 1), token 8 q + 2 t + (i & 1))
    constexpr int TILE_F = 2 * TG * 32 * 4;
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const uint32_t crank = cluster_rank();
    const int C = p.C;
    const int cluster_id = static_cast<int>(blockIdx.x) / C, nclusters = static_cast<int>(gridDim.x) / C;
    const int S = p.stages;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem) + warp * kBMaxStages;
    float *sq = reinterpret_cast<float *>(smem + 512);                 // [C][kBMaxTokens]
    float *recv = reinterpret_cast<float *>(smem + 512 + kBMaxC * kBMaxTokens * 4);  // [8][TILE_F]
    uint8_t *xs = smem + p.off_x;
    uint8_t *xsum = xs + T * p.xrow;
    uint8_t *stages = smem + p.off_stage + static_cast<size_t>(warp) * S * kBStage;
    const int nsb = p.kc >> 8;
    const int sb0 = static_cast<int>(crank) * nsb;
    const int ucount = cluster_id < p.units ? (p.units - cluster_id + nclusters - 1) / nclusters : 0;

    // item i of this warp: unit (cluster_id + (i / nsb) * nclusters), super-block sb0 + i % nsb
    auto item_tile = [&](int i) { return b_tile(p, (static_cast<int64_t>(cluster_id) + (i / nsb) * nclusters) * 8 + warp); };
    int ahead = 0;
    const int nitems = ucount * nsb;
    if (lane == 0) {
        for (int i = 0; i < S; ++i) mbar_init(&full[i], 1);
        fence_mbar_init();
        for (; ahead < S && ahead < nitems; ++ahead) {
            const BTile tl = item_tile(ahead);
            if (tl.valid) b_issue(p, tl, sb0 + ahead % nsb, stages + static_cast<size_t>(ahead) * kBStage, &full[ahead]);
        }
    }
    ahead = __shfl_sync(0xffffffffu, ahead, 0);
    __syncwarp();
    pdl_wait();
    pdl_trigger();
    // every CTA of the cluster must be running before distributed shared memory is written
    cl_arrive();
    cl_wait();
    bx_prepare<T>(p, crank, xs, xsum, sq, recv);

    const uint32_t xs_a = smem_u32(xs), xsum_a = smem_u32(xsum), st_a = smem_u32(stages);
    int s = 0;
    uint32_t phase = 0;
    bool failed = false;
    int item = 0;
    for (int ui = 0; ui < ucount; ++ui) {
        const int64_t unit = static_cast<int64_t>(cluster_id) + static_cast<int64_t>(ui) * nclusters;
        const BTile tl = b_tile(p, unit * 8 + warp);
        float acc[2][TG][4];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int q = 0; q < TG; ++q)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[h][q][i] = 0.0f;
        for (int jb = 0; jb < nsb; ++jb, ++item) {
            if (tl.valid) {
                if (!failed && !mbar_wait(&full[s], phase)) {
                    report_device_error(T2C_ETIMEOUT);
                    failed = true;
                }
                if (!failed)
                    b_block<TG>(st_a + static_cast<uint32_t>(s * kBStage), xs_a, xsum_a, p.xrow, nsb, jb, lane, acc);
                __syncwarp();
            }
            // refill this stage with the item S ahead (only items of existing tiles take a stage)
            if (tl.valid) {
                if (ahead < nitems) {
                    const BTile nt = item_tile(ahead);
                    if (lane == 0 && nt.valid && !failed) {
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        b_issue(p, nt, sb0 + ahead % nsb, stages + static_cast<size_t>(s) * kBStage, &full[s]);
                    }
                    ++ahead;
                }
                if (++s == S) {
                    s = 0;
                    phase ^= 1u;
                }
            }
        }
        // partial tile -> owner CTA (warp % C), slot (warp / C) * C + crank
        if (ui > 0) cl_wait();  // the owner finished reading the previous unit's partials
        if (tl.valid) {
            const uint32_t owner = static_cast<uint32_t>(warp % C);
            float *slot = recv + ((warp / C) * C + static_cast<int>(crank)) * TILE_F;
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int q = 0; q < TG; ++q)
                    st_cluster_v4(slot + ((h * TG + q) * 32 + lane) * 4, owner, acc[h][q][0], acc[h][q][1],
                                  acc[h][q][2], acc[h][q][3]);
        }
        cl_arrive();
        cl_wait();
        // owned tiles of the unit: warps w with w % C == crank (at most 8 / C = 2 with C >= 4); thread
        // (part, lane) adds 4 values of the C slots in rank order.  The sums go to registers first: the
        // receive buffer is released before the output stores, so those drain while the next unit computes
        // instead of holding up the next release (the release then waits only for stores long done).
        constexpr int kOwn = 2;
        float ov[kOwn][2][4];
        int own_w[kOwn];
        const int part = threadIdx.x >> 5;
        const int nparts = p.swiglu ? TG : 2 * TG;
#pragma unroll
        for (int o = 0; o < kOwn; ++o) {
            own_w[o] = static_cast<int>(crank) + o * C;
#pragma unroll
            for (int r = 0; r < 2; ++r)
#pragma unroll
                for (int i = 0; i < 4; ++i) ov[o][r][i] = 0.0f;
            if (own_w[o] >= kBWarps || part >= nparts) continue;
            const float *base = recv + (own_w[o] / C) * C * TILE_F;
            for (int c = 0; c < C; ++c) {
                const float4 a = *reinterpret_cast<const float4 *>(base + c * TILE_F + (part * 32 + lane) * 4);
                ov[o][0][0] += a.x;
                ov[o][0][1] += a.y;
                ov[o][0][2] += a.z;
                ov[o][0][3] += a.w;
                if (p.swiglu) {  // part q (gate rows) with part TG + q (up rows)
                    const float4 b =
                        *reinterpret_cast<const float4 *>(base + c * TILE_F + ((TG + part) * 32 + lane) * 4);
                    ov[o][1][0] += b.x;
                    ov[o][1][1] += b.y;
                    ov[o][1][2] += b.z;
                    ov[o][1][3] += b.w;
                }
            }
        }
        cl_arrive();
        const int lg = lane >> 2, lt = lane & 3;
#pragma unroll
        for (int o = 0; o < kOwn; ++o) {
            if (own_w[o] >= kBWarps || part >= nparts) continue;
            const BTile ot = b_tile(p, unit * 8 + own_w[o]);
            if (!ot.valid) continue;
            if (p.swiglu) {
                const int64_t n = p.n[0];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int64_t row = ot.row0 + lg + 8 * (i >> 1);
                    const int tok = 8 * part + 2 * lt + (i & 1);
                    if (row < n && tok < p.M)
                        p.y[0][static_cast<int64_t>(tok) * n + row] = __float2half_rn(silu_b(ov[o][0][i]) * ov[o][1][i]);
                }
            } else {
                const int h = part / TG, q = part - h * TG;
                const int64_t n = p.n[ot.si];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int64_t row = ot.row0 + 16 * h + lg + 8 * (i >> 1);
                    const int tok = 8 * q + 2 * lt + (i & 1);
                    if (row >= n || tok >= p.M) continue;
                    const int64_t oi = static_cast<int64_t>(tok) * n + row;
                    float val = ov[o][0][i];
                    if (p.res[ot.si] != nullptr) val += __half2float(p.res[ot.si][oi]);
                    p.y[ot.si][oi] = __float2half_rn(val);
                }
            }
        }
    }
    // the last arrive's partner wait: no CTA leaves while another may still address its shared memory
    if (ucount > 0) cl_wait();
}

int encode_map_b(CUtensorMap *map, const uint8_t *w, int64_t n, int64_t row_bytes) {
    static PFN_cuTensorMapEncodeTiled encode = [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            fn = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled>(fn);
    }();
    if (encode == nullptr || row_bytes % 16 != 0 || reinterpret_cast<uintptr_t>(w) % 16 != 0) return T2C_EUNSUPPORTED;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes / 4), static_cast<cuuint64_t>(n)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
    const cuuint32_t box[2] = {36, 16};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint8_t *>(w), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? T2C_OK : T2C_EUNSUPPORTED;
}

template <int TG>
int launch_tg(BParams p, int M, cudaStream_t stream) {
    static bool configured[64] = {false};
    constexpr int T = 8 * TG;
    p.M = M;
    p.xrow = bx_row_bytes(p.kc);
    const size_t recv_end = 512 + kBMaxC * kBMaxTokens * 4 + static_cast<size_t>(8) * 2 * TG * 32 * 4 * 4;
    p.off_x = (recv_end + 127) / 128 * 128;
    const size_t xbytes = static_cast<size_t>(T) * p.xrow + static_cast<size_t>(T) * (p.kc / 256) * 32;
    p.off_stage = (p.off_x + xbytes + 1023) / 1024 * 1024;
    const size_t per_stage = static_cast<size_t>(kBWarps) * kBStage;
    if (p.off_stage + 2 * per_stage > kBSmemLimit) return T2C_EUNSUPPORTED;
    p.stages = static_cast<int>((kBSmemLimit - p.off_stage) / per_stage);
    if (p.stages > kBMaxStages) p.stages = kBMaxStages;
    const size_t smem = p.off_stage + per_stage * p.stages;
    int device = 0;
    cudaGetDevice(&device);
    const int slot = device < 0 ? 0 : (device > 63 ? 63 : device);
    if (!configured[slot]) {
        if (cudaFuncSetAttribute(qbatch_kernel<TG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem < kBSmemLimit ? kBSmemLimit : smem)) != cudaSuccess)
            return set_error(T2C_ECUDA, "qbatch: cudaFuncSetAttribute failed");
        configured[slot] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kBThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = static_cast<unsigned>(p.C);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    // persistent clusters: as many as fit at once, at most one per unit
    cfg.gridDim = dim3(static_cast<unsigned>(p.C));
    int max_clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&max_clusters, qbatch_kernel<TG>, &cfg) != cudaSuccess || max_clusters < 1)
        max_clusters = sm_count() / p.C;
    if (max_clusters < 1) return T2C_EUNSUPPORTED;
    const int nclusters = p.units < max_clusters ? p.units : max_clusters;
    cfg.gridDim = dim3(static_cast<unsigned>(nclusters * p.C));
    const cudaError_t err = cudaLaunchKernelEx(&cfg, qbatch_kernel<TG>, p);
    if (err != cudaSuccess) return set_error(T2C_ECUDA, "qbatch launch: %s", cudaGetErrorString(err));
    return T2C_OK;
}

}  // namespace

// 5.. tokens of Q4_K linears (ROWS with up to 3 weights, or SWIGLU), chunked
// by 16 tokens per launch (the dispatcher sends it 5..16 tokens).  T2C_EUNSUPPORTED when the call is not served
// (another type, argmax, fp32 outputs, bias or activation, K % 256 != 0).
int qbatch(const QGemmArgs &a, const float *norm_w, float eps, cudaStream_t stream) {
    if (a.M < 5 || a.K % 256 != 0 || a.K > 65536 || a.ps != nullptr || a.bias != nullptr || a.act != 0)
        return T2C_EUNSUPPORTED;
    const bool swiglu = a.w_up != nullptr;
    if (a.fmt != T2C_Q4_K || (swiglu && a.nw != 1)) return T2C_EUNSUPPORTED;
    for (int i = 0; i < a.nw; ++i)
        if (a.yf[i] != nullptr || a.w[i] == nullptr || a.y[i] == nullptr) return T2C_EUNSUPPORTED;
    if (reinterpret_cast<uintptr_t>(a.x) % 16 != 0 || (norm_w && reinterpret_cast<uintptr_t>(norm_w) % 16 != 0))
        return T2C_EUNSUPPORTED;
    BParams p = {};
    const int64_t row_bytes = a.K / 256 * 144;
    p.swiglu = swiglu ? 1 : 0;
    p.nstreams = swiglu ? 1 : a.nw;
    int64_t tiles = 0;
    if (swiglu) {
        if (encode_map_b(&p.tmap[0], a.w[0], a.N[0], row_bytes) || encode_map_b(&p.tmap[1], a.w_up, a.N[0], row_bytes))
            return T2C_EUNSUPPORTED;
        p.n[0] = a.N[0];
        p.tile_begin[0] = 0;
        tiles = (a.N[0] + 15) / 16;
        p.tile_begin[1] = tiles;
    } else {
        for (int i = 0; i < a.nw; ++i) {
            if (encode_map_b(&p.tmap[i], a.w[i], a.N[i], row_bytes)) return T2C_EUNSUPPORTED;
            p.n[i] = a.N[i];
            p.tile_begin[i] = tiles;
            tiles += (a.N[i] + kBRows - 1) / kBRows;
        }
        p.tile_begin[a.nw] = tiles;
    }
    for (int i = p.nstreams + 1; i < 4; ++i) p.tile_begin[i] = tiles;
    p.units = static_cast<int>((tiles + kBWarps - 1) / kBWarps);
    const int nsb_total = static_cast<int>(a.K / 256);
    int C = kBMaxC;
    while (C > 1 && nsb_total % C) C >>= 1;
    if (C < 4) return T2C_EUNSUPPORTED;  // a CTA owns at most two tiles of a unit
    p.C = C;
    p.kc = static_cast<int>(a.K / C);
    p.K = static_cast<int>(a.K);
    p.norm_w = norm_w;
    p.eps = eps;
    for (int64_t m0 = 0; m0 < a.M; m0 += kBMaxTokens) {
        const int m = static_cast<int>((a.M - m0) < kBMaxTokens ? (a.M - m0) : kBMaxTokens);
        BParams c = p;
        c.x = a.x + m0 * a.K;
        for (int i = 0; i < a.nw; ++i) {
            c.y[i] = a.y[i] + m0 * a.N[i];
            c.res[i] = a.res[i] ? a.res[i] + m0 * a.N[i] : nullptr;
        }
        const int rc = m <= 8 ? launch_tg<1>(c, m, stream) : launch_tg<2>(c, m, stream);
        if (rc != T2C_OK) return rc;
    }
    return T2C_OK;
}

cudaError_t status_qbatch(unsigned int *bits, int clear, cudaStream_t s) { return read_tu_status(bits, clear, s); }

}  // namespace t2c
