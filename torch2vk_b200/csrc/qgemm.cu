// Q4_K / Q6_K / Q8_0 GEMM on tcgen05 tensor cores with TMEM accumulators (M > 4 tokens:
// prefill, batched decode).  The weights are the A operand: a CTA owns 128
// weight rows (UMMA M = 128) and mt tokens (UMMA N = mt, <= 256), so
//   D[n, m] = sum_k deq(W)[n, k] * x[m, k]     (fp32 in TMEM, 128 lanes x mt columns)
// and the epilogue writes y[m, n] (+ residual) or silu(gate) * up.
//
// Per K chunk of 64 values (one 128-byte row of a 128B-swizzled K-major atom):
//  * raw Q4_K super-blocks of the 128 rows arrive by 2-D TMA (box 144 B x 128
//    rows, two stages; requested before griddepcontrol.wait: weights are static);
//  * x[mt, 64] fp16 arrives by 2-D TMA with 128-byte swizzle (three buffers,
//    two chunks ahead);
//  * 8 warps dequantize (two threads per row, one 32-value sub-block each),
//    d*sc*q - dmin*m in fp32 rounded to fp16, straight into the swizzled
//    K-major A layout (three buffers);
//  * one thread of the issue warp issues 4 x tcgen05.mma kind::f16 (K = 16
//    each) and commits them to the buffer's mbarrier, which also tells when
//    A / x may be reused; one thread of the producer warp issues the TMA copies.
// Descriptors (PTX ISA "shared memory descriptor" / "instruction descriptor"):
// K-major SWIZZLE_128B: start >> 4, LBO 1, SBO 1024 >> 4, version 1, layout 2;
// a K step of 16 fp16 advances the start address by 32 bytes.
// When (row tile, token tile) pairs are too few to fill the GPU (small M), a
// cluster of up to 8 CTAs splits K; each parks its fp32 partials in its own
// shared memory and the cluster leader sums them over distributed shared
// memory (mapa / ld.shared::cluster) before the epilogue.
// Every wait is bounded; on a timeout the kernel reports T2C_ETIMEOUT, stops
// issuing, frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "qgemm.cuh"

namespace t2c {
namespace {

constexpr int kRowsT = 128;                 // weight rows per CTA (UMMA M)
constexpr int kKC = 64;                     // values per K chunk
constexpr int kNB = 3;                      // A / x buffers
// Raw weight stage = one 256-value block of 128 rows.  Q4_K: 144-byte blocks,
// box 36 u32.  Q6_K: 210-byte blocks start at even, not 16-byte aligned,
// offsets, so the box is the 224-byte window from the 16-byte boundary at or
// below the block start (the block sits at offset (210 b) % 16 in it).
template <int FMT>
struct RawFmt;
template <>
struct RawFmt<T2C_Q4_K> {
    static constexpr int kRow = 144, kBox = 36;
    __device__ static int x_of(int b) { return b * 36; }
    __device__ static int off_of(int) { return 0; }
};
// When K % 2048 != 0 a Q6_K row is not a multiple of 16 bytes, so no 2-D map
// can step from row to row; eight rows always are (8 x 210 x K / 256 bytes).
// Grouped mode then maps the weight as [N / 8 groups, 8 rows' bytes] and a
// stage is eight boxes of 16 groups x 224 bytes, box j holding row j of every
// group: weight row r = 8 g + j lands in stage slot 16 j + g, at offset
// (j x row_bytes + 210 b) % 16 within its 224-byte window.
template <>
struct RawFmt<T2C_Q6_K> {
    static constexpr int kRow = 224, kBox = 56;
    __device__ static int x_of(int b) { return ((210 * b) >> 4) * 4; }
    __device__ static int off_of(int b) { return (210 * b) & 15; }
    __device__ static int gx_of(int b, int j, int row_bytes) { return ((j * row_bytes + 210 * b) >> 4) * 4; }
    __device__ static int goff_of(int b, int j, int row_bytes) { return (j * row_bytes + 210 * b) & 15; }
};
// Q8_0: 34-byte blocks of 32 values; eight of them (272 bytes, a multiple of 16) make the
// 256-value group of a raw stage, so the TMA window starts on a 16-byte boundary.
template <>
struct RawFmt<T2C_Q8_0> {
    static constexpr int kRow = 272, kBox = 68;
    __device__ static int x_of(int b) { return b * 68; }
    __device__ static int off_of(int) { return 0; }
};
constexpr int kRawBytesMax = kRowsT * 272;
constexpr int kABytes = kRowsT * kKC * 2;   // 16 KB of fp16
constexpr int kDeqWarps = 8;                // dequantization warps (2 threads per weight row)
constexpr int kIssuer = 8;                  // warp that issues the tcgen05 MMAs
constexpr int kProducer = 9;                // warp that issues the TMA copies
constexpr int kThreadsG = 32 * (kDeqWarps + 2);

struct GemmParams {
    alignas(64) CUtensorMap wmap[3];  // raw Q4_K words [N, row_bytes / 4], box 36 x 128, per weight
    alignas(64) CUtensorMap umap;     // up weight (SwiGLU)
    alignas(64) CUtensorMap xmap;     // x fp16 [M, K], box 64 x mt, 128-byte swizzle
    __half *y[3];
    float *yf[3];                     // fp32 outputs instead of y (non-null), plain linear only
    const __half *res[3];
    int64_t Nw[3];
    int tile0[4];                     // first row tile of each weight (tile0[nw] = all row tiles)
    int nw;
    int64_t M;
    int K, mt, swiglu, tmem_cols;
    int ksplit;  // CTAs of a cluster splitting K (1: no split)
    float *ps;   // argmax mode: best (score, row) per group of 4 rows, [M, G]
    uint32_t *pt;
    int64_t G;
    const float *bias;  // plain single-weight mode: fp32 [N] added before the activation
    int act;            // 1: erf GELU
    int q6_grouped;     // Q6_K rows of K % 2048 != 0: eight-row group maps (RawFmt<T2C_Q6_K>)
    int row_bytes;
    int stacked;        // SwiGLU at small token tiles: a CTA's 128 A rows are 64 gate rows over the same 64 up rows
};

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1u) << 16) |
           (static_cast<uint64_t>(1024u >> 4) << 32) | (static_cast<uint64_t>(1u) << 46) |
           (static_cast<uint64_t>(2u) << 61);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, bool acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc ? 1u : 0u)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t v[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float gelu_erf_g(float v) { return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f)); }

__device__ __forceinline__ float small_u2f_g(uint32_t v) { return __uint_as_float(0x4B000000u | v) - 8388608.0f; }

// One sub-block half of a 64-value chunk: row r of quarter q of a 144-byte
// Q4_K block, nibble half hf (0: low nibbles = values 0..31 of the chunk,
// sub-block 2q; 1: high nibbles = values 32..63, sub-block 2q + 1) -> four
// swizzled 16-byte chunks (4 hf .. 4 hf + 3) of fp16 d * (sc q) - dmin m.
// Two nibbles at a time become the fp16 pair 1024 + q (byte_perm into
// 0x64xx); one paired fma gives sc q exactly (an integer <= 945), a second
// one d * (sc q) - dmin m with the fp16 super-block scale d, so the only
// roundings are that of dmin m (formed in fp32) and the final one.
__device__ __forceinline__ uint32_t nib_pair(uint32_t src, uint32_t sel, __half2 sc2, __half2 nb2, __half2 d2,
                                             __half2 ndm2) {
    const uint32_t u = __byte_perm(src, 0x64646464u, sel);
    const __half2 qs = __hfma2(*reinterpret_cast<const __half2 *>(&u), sc2, nb2);
    const __half2 v = __hfma2(d2, qs, ndm2);
    return *reinterpret_cast<const uint32_t *>(&v);
}

__device__ __forceinline__ void dequant_half(const uint8_t *raw_row, int q, int hf, uint32_t a_row, int r) {
    const uint4 h = *reinterpret_cast<const uint4 *>(raw_row);
    const uint4 n0 = *reinterpret_cast<const uint4 *>(raw_row + 16 + 32 * q);
    const uint4 n1 = *reinterpret_cast<const uint4 *>(raw_row + 32 + 32 * q);
    // 6-bit codes of sub-block j = 2q + hf (packing of quantize/vulkan.py:331-342)
    const int j = 2 * q + hf, jb = j & 3;
    const uint32_t y = (h.y >> (8 * jb)) & 0xffu, z = (h.z >> (8 * jb)) & 0xffu, w = (h.w >> (8 * jb)) & 0xffu;
    const uint32_t sc = j < 4 ? (y & 63u) : ((w & 15u) | ((y >> 6) << 4));
    const uint32_t mn = j < 4 ? (z & 63u) : ((w >> 4) | ((z >> 6) << 4));
    const float scf = small_u2f_g(sc);
    const __half2 sc2 = __float2half2_rn(scf), nb2 = __float2half2_rn(-1024.0f * scf);
    const uint32_t dbits = (h.x & 0xffffu) * 0x10001u;
    const __half2 d2 = *reinterpret_cast<const __half2 *>(&dbits);
    const __half2 ndm2 = __float2half2_rn(-(half_bits_to_float(h.x >> 16) * small_u2f_g(mn)));
    const uint32_t wq[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
    const int sh = 4 * hf;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        // values 8c .. 8c+7 of the sub-block = nibble hf of bytes 8c .. 8c+7 of the quarter
        const uint32_t lo = (wq[2 * c] >> sh) & 0x0F0F0F0Fu, hi = (wq[2 * c + 1] >> sh) & 0x0F0F0F0Fu;
        const uint32_t p0 = nib_pair(lo, 0x4140u, sc2, nb2, d2, ndm2), p1 = nib_pair(lo, 0x4342u, sc2, nb2, d2, ndm2);
        const uint32_t p2 = nib_pair(hi, 0x4140u, sc2, nb2, d2, ndm2), p3 = nib_pair(hi, 0x4342u, sc2, nb2, d2, ndm2);
        const uint32_t dst = a_row + static_cast<uint32_t>((((4 * hf + c) ^ (r & 7)) << 4));
        asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(dst), "r"(p0), "r"(p1), "r"(p2), "r"(p3) : "memory");
    }
}

// 4 bytes at a 2-byte aligned shared address a, as aligned words w[i] = bytes a + 4 i .. (i < n).
template <int N>
__device__ __forceinline__ void lds_words_a2(uint32_t a, uint32_t w[N]) {
    const uint32_t base = a & ~3u, sh = (a & 3u) * 8u;
    uint32_t r[N + 1];
#pragma unroll
    for (int i = 0; i <= N; ++i) asm volatile("ld.shared.u32 %0, [%1];" : "=r"(r[i]) : "r"(base + 4 * i));
#pragma unroll
    for (int i = 0; i < N; ++i) w[i] = __funnelshift_r(r[i], r[i + 1], sh);
}

// Q6_K: chunk ch (values 64 ch .. 64 ch + 63) of the 210-byte block at shared
// address blk (2-byte aligned), half hf -> four swizzled 16-byte chunks of
// fp16 (d * sc) * (q - 32), formed in fp32 as the reference decoder does
// (linear_nobias_q6_k_matvec_f32.py:116-156): value l of group c = 2 (ch & 1)
// + hf of half-block s = ch >> 1 has its low 4 bits in nibble (ch & 1) of
// ql[64 s + 32 hf + l], its high 2 bits at bit 2c of qh[32 s + l], and scale
// sc[8 s + 2 c + l / 16].
__device__ __forceinline__ void dequant_q6k_half(uint32_t blk, int ch, int hf, uint32_t a_row, int r) {
    const int s = ch >> 1, c = 2 * (ch & 1) + hf;
    uint32_t ql[8], qh[8], sw[1], dw[1];
    lds_words_a2<8>(blk + 64 * s + 32 * hf, ql);
    lds_words_a2<8>(blk + 128 + 32 * s, qh);
    lds_words_a2<1>(blk + 192 + 8 * s + 2 * c, sw);
    lds_words_a2<1>(blk + 208, dw);
    const float d = half_bits_to_float(dw[0]);
    const float ds0 = d * static_cast<float>(static_cast<int8_t>(sw[0] & 0xffu));
    const float ds1 = d * static_cast<float>(static_cast<int8_t>((sw[0] >> 8) & 0xffu));
    const int nsh = 4 * (ch & 1), hsh = 2 * c;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float ds = j < 2 ? ds0 : ds1;
        uint32_t packed[4];
#pragma unroll
        for (int wi = 0; wi < 2; ++wi) {
            const uint32_t qv = ((ql[2 * j + wi] >> nsh) & 0x0F0F0F0Fu) | (((qh[2 * j + wi] >> hsh) & 0x03030303u) << 4);
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const float v0 = ds * (__uint_as_float(__byte_perm(qv, 0x4B000000u, 0x7440u + 2 * e)) - 8388640.0f);
                const float v1 = ds * (__uint_as_float(__byte_perm(qv, 0x4B000000u, 0x7441u + 2 * e)) - 8388640.0f);
                const __half2 hv = __floats2half2_rn(v0, v1);
                packed[2 * wi + e] = *reinterpret_cast<const uint32_t *>(&hv);
            }
        }
        const uint32_t dst = a_row + static_cast<uint32_t>((((4 * hf + j) ^ (r & 7)) << 4));
        asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(dst), "r"(packed[0]), "r"(packed[1]),
                     "r"(packed[2]), "r"(packed[3])
                     : "memory");
    }
}

// Q8_0: chunk q (values 64 q .. 64 q + 63) of the 272-byte group of 8 blocks at shared address
// grp, half hf = block 2 q + hf -> four swizzled 16-byte chunks of fp16 d * q.  Each int8 becomes
// the exact fp16 integer q ((1024 + (q + 128)) - 1152, byte_perm into 0x64xx), and one paired
// multiply by the fp16 block scale d gives the only rounding (the reference forms d * q in fp32:
// linear_nobias_q8_0_matvec_f32.py:84-95).
__device__ __forceinline__ void dequant_q8_half(uint32_t grp, int q, int hf, uint32_t a_row, int r) {
    const uint32_t blk = grp + 34u * static_cast<uint32_t>(2 * q + hf);
    uint32_t w[8], dw[1];
    lds_words_a2<8>(blk + 2, w);
    lds_words_a2<1>(blk, dw);
    const uint32_t dbits = (dw[0] & 0xffffu) * 0x10001u;
    const __half2 d2 = *reinterpret_cast<const __half2 *>(&dbits);
    const __half2 off = __float2half2_rn(1152.0f);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        uint32_t packed[4];
#pragma unroll
        for (int wi = 0; wi < 2; ++wi) {
            const uint32_t u = w[2 * c + wi] ^ 0x80808080u;  // q + 128 per byte
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const uint32_t hv = __byte_perm(u, 0x64646464u, e ? 0x4342u : 0x4140u);
                const __half2 qv = __hsub2(*reinterpret_cast<const __half2 *>(&hv), off);
                const __half2 v = __hmul2(qv, d2);
                packed[2 * wi + e] = *reinterpret_cast<const uint32_t *>(&v);
            }
        }
        const uint32_t dst = a_row + static_cast<uint32_t>((((4 * hf + c) ^ (r & 7)) << 4));
        asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(dst), "r"(packed[0]), "r"(packed[1]),
                     "r"(packed[2]), "r"(packed[3])
                     : "memory");
    }
}

// Argmax epilogue: for token m, the best (value, row) of each group of 4 rows
// (four consecutive lanes; ties keep the lower row) -> ps / pt[m, n / 4].
__device__ __forceinline__ void argmax4_store(const GemmParams &p, int64_t m, int64_t n, int64_t N, float v, bool ok) {
    float best = (n < N && ok) ? v : -INFINITY;
    uint32_t tok = static_cast<uint32_t>(n);
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const uint32_t ot = __shfl_xor_sync(0xffffffffu, tok, o);
        if (ob > best || (ob == best && ot < tok)) {
            best = ob;
            tok = ot;
        }
    }
    if ((n & 3) == 0 && n < N && m < p.M) {
        p.ps[m * p.G + (n >> 2)] = best;
        p.pt[m * p.G + (n >> 2)] = tok;
    }
}

// Sum over the ks ranks of a cluster (rank order) of four consecutive fp32 partials at byte
// offset off of each rank's parked buffer (rbase: the ranks' DSMEM addresses; ks == 1: this
// CTA's own shared memory).  All loads are issued before the first add.
__device__ __forceinline__ void sum_parked(const uint32_t rbase[8], int ks, uint32_t off, float out[4]) {
    float v[8][4];
#pragma unroll
    for (int rk = 0; rk < 8; ++rk) {
        if (rk < ks) {
            if (ks > 1)
                asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
                             : "=f"(v[rk][0]), "=f"(v[rk][1]), "=f"(v[rk][2]), "=f"(v[rk][3])
                             : "r"(rbase[rk] + off));
            else
                asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                             : "=f"(v[rk][0]), "=f"(v[rk][1]), "=f"(v[rk][2]), "=f"(v[rk][3])
                             : "r"(rbase[rk] + off));
        }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) out[j] = 0.0f;
#pragma unroll
    for (int rk = 0; rk < 8; ++rk)
        if (rk < ks) {
#pragma unroll
            for (int j = 0; j < 4; ++j) out[j] += v[rk][j];
        }
}

// Warp roles: warps 0..7 dequantize (thread = weight row tid % 128, nibble
// half tid / 128), warp 8 issues the MMAs, warp 9 issues the TMA copies.
// They meet only at mbarriers: raw_full / raw_empty (raw weight stages),
// x_full (x chunks), a_full (dequantized A buffers, one arrival per dequant
// warp) and mma_done (tcgen05.commit: A / x buffer free again).
template <int FMT>
__global__ void __launch_bounds__(kThreadsG, 2) qgemm_kernel(const __grid_constant__ GemmParams p) {
    using RF = RawFmt<FMT>;
    constexpr int kRawBytes = kRowsT * RF::kRow;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled operand tiles
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mt = p.mt;
    const bool swiglu = p.swiglu != 0;
    const int kpart = blockIdx.x % p.ksplit;  // rank in the cluster
    // row tile -> weight (fused QKV: consecutive tile ranges of the three weights)
    const int tile = static_cast<int>(blockIdx.x / p.ksplit);
    int wi = 0;
    if (p.nw > 1 && tile >= p.tile0[1]) wi = (p.nw > 2 && tile >= p.tile0[2]) ? 2 : 1;
    const bool stacked = p.stacked != 0;
    const int64_t n0 = static_cast<int64_t>(tile - p.tile0[wi]) * (stacked ? kRowsT / 2 : kRowsT);
    const CUtensorMap *wmap = &p.wmap[wi];
    __half *const yout = p.y[wi];
    float *const youtf = p.yf[wi];
    const __half *const res = p.res[wi];
    const int64_t N = p.Nw[wi];
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * mt;
    const int nsb = p.K / 256 / p.ksplit;  // super-blocks of this CTA's K range
    const int sb0 = kpart * nsb;
    const int nch = nsb * 4, kc0 = sb0 * 4;
    const int xbytes = mt * 128;

    uint8_t *ptr = smem;
    const uint32_t a_base = smem_u32(ptr);
    ptr += kNB * kABytes;
    const uint32_t aup_base = smem_u32(ptr);
    if (swiglu) ptr += kNB * kABytes;
    uint8_t *x_ptr = ptr;
    const uint32_t x_base = smem_u32(ptr);
    ptr += kNB * xbytes;
    uint8_t *raw_ptr = ptr;
    ptr += 2 * kRawBytes;
    uint8_t *rawup_ptr = ptr;
    if (swiglu) ptr += 2 * kRawBytes;
    uint64_t *raw_full = reinterpret_cast<uint64_t *>(ptr);
    uint64_t *raw_empty = raw_full + 2;
    uint64_t *x_full = raw_empty + 2;
    uint64_t *a_full = x_full + kNB;
    uint64_t *mma_done = a_full + kNB;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + kNB);
    __shared__ int failed_s;
    volatile int &failed = failed_s;
    const uint32_t raw_bytes = swiglu ? 2u * kRawBytes : static_cast<uint32_t>(kRawBytes);
    // raw weight stage s <- super-block sb (absolute); the caller has armed raw_full[s]
    auto load_raw = [&](int s, int sb) {
        if constexpr (FMT == T2C_Q6_K) {
            if (p.q6_grouped) {
#pragma unroll 1
                for (int j = 0; j < 8; ++j)
                    tma_load_2d(raw_ptr + s * kRawBytes + j * 16 * RF::kRow, wmap, RF::gx_of(sb, j, p.row_bytes),
                                static_cast<int>(n0 >> 3), &raw_full[s]);
                return;
            }
        }
        if (stacked) {
            // gate rows n0 .. n0 + 63 over up rows n0 .. n0 + 63 (64-row boxes)
            tma_load_2d(raw_ptr + s * kRawBytes, wmap, RF::x_of(sb), static_cast<int>(n0), &raw_full[s]);
            tma_load_2d(raw_ptr + s * kRawBytes + (kRowsT / 2) * RF::kRow, &p.umap, RF::x_of(sb), static_cast<int>(n0),
                        &raw_full[s]);
            return;
        }
        tma_load_2d(raw_ptr + s * kRawBytes, wmap, RF::x_of(sb), static_cast<int>(n0), &raw_full[s]);
        if (swiglu) tma_load_2d(rawup_ptr + s * kRawBytes, &p.umap, sb * 36, static_cast<int>(n0), &raw_full[s]);
    };

    if (tid == kProducer * 32) {
        failed = 0;
        for (int i = 0; i < 2; ++i) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], kDeqWarps);
        }
        for (int i = 0; i < kNB; ++i) {
            mbar_init(&x_full[i], 1);
            mbar_init(&a_full[i], kDeqWarps);
            mbar_init(&mma_done[i], 1);
        }
        fence_mbar_init();
        // static weights: first two super-blocks before the dependency on the previous kernel
        for (int s = 0; s < 2 && s < nsb; ++s) {
            mbar_arrive_expect_tx(&raw_full[s], raw_bytes);
            load_raw(s, sb0 + s);
        }
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(static_cast<uint32_t>(p.tmem_cols))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(tmem_slot);
    pdl_wait();
    pdl_trigger();

    if (warp == kProducer) {
        if (lane == 0) {
            for (int c = 0; c < kNB - 1 && c < nch; ++c) {
                mbar_arrive_expect_tx(&x_full[c], static_cast<uint32_t>(xbytes));
                tma_load_2d(x_ptr + c * xbytes, &p.xmap, (kc0 + c) * kKC, static_cast<int>(m0), &x_full[c]);
            }
            for (int kc = 0; kc < nch && !failed; ++kc) {
                // x of chunk kc + kNB - 1 goes into the buffer of chunk kc - 1 once its MMAs are done
                const int nx = kc + kNB - 1;
                if (nx < nch) {
                    const int bx = nx % kNB;
                    if (kc >= 1 && !mbar_wait(&mma_done[bx], static_cast<uint32_t>(((kc - 1) / kNB) & 1))) {
                        failed = 1;
                        break;
                    }
                    mbar_arrive_expect_tx(&x_full[bx], static_cast<uint32_t>(xbytes));
                    tma_load_2d(x_ptr + bx * xbytes, &p.xmap, (kc0 + nx) * kKC, static_cast<int>(m0), &x_full[bx]);
                }
                // raw stage of super-block sb is free after its last quarter: load sb + 2
                if ((kc & 3) == 3) {
                    const int sb = kc >> 2;
                    if (sb + 2 < nsb) {
                        if (!mbar_wait(&raw_empty[sb & 1], static_cast<uint32_t>((sb >> 1) & 1))) {
                            failed = 1;
                            break;
                        }
                        mbar_arrive_expect_tx(&raw_full[sb & 1], raw_bytes);
                        load_raw(sb & 1, sb0 + sb + 2);
                    }
                }
            }
        }
    } else if (warp == kIssuer) {
        if (lane == 0) {
            const uint32_t idesc =
                (1u << 4) | (static_cast<uint32_t>(mt >> 3) << 17) | (static_cast<uint32_t>(kRowsT >> 4) << 24);
            for (int kc = 0; kc < nch && !failed; ++kc) {
                const int b = kc % kNB;
                const uint32_t ph = static_cast<uint32_t>((kc / kNB) & 1);
                if (!mbar_wait(&a_full[b], ph) || !mbar_wait(&x_full[b], ph)) {
                    failed = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t xa = x_base + static_cast<uint32_t>(b * xbytes);
                const uint32_t aa = a_base + static_cast<uint32_t>(b * kABytes);
#pragma unroll
                for (int s = 0; s < kKC / 16; ++s)
                    umma_f16(tmem, sw128_desc(aa + 32 * s), sw128_desc(xa + 32 * s), idesc, kc > 0 || s > 0);
                if (swiglu) {
                    const uint32_t au = aup_base + static_cast<uint32_t>(b * kABytes);
#pragma unroll
                    for (int s = 0; s < kKC / 16; ++s)
                        umma_f16(tmem + static_cast<uint32_t>(mt), sw128_desc(au + 32 * s), sw128_desc(xa + 32 * s),
                                 idesc, kc > 0 || s > 0);
                }
                umma_commit(&mma_done[b]);
            }
        }
    } else {
        // dequantization warps
        const int r = tid & (kRowsT - 1), hf = tid >> 7;
        for (int kc = 0; kc < nch; ++kc) {
            const int sb = kc >> 2, q = kc & 3, b = kc % kNB;
            bool ok = true;
            if (q == 0) ok = mbar_wait(&raw_full[sb & 1], static_cast<uint32_t>((sb >> 1) & 1));
            if (ok && kc >= kNB) ok = mbar_wait(&mma_done[b], static_cast<uint32_t>(((kc - kNB) / kNB) & 1));
            if (!ok || failed) {
                failed = 1;
                break;
            }
            if constexpr (FMT == T2C_Q8_0) {
                dequant_q8_half(smem_u32(raw_ptr + (sb & 1) * kRawBytes + r * RF::kRow), q, hf,
                                a_base + static_cast<uint32_t>(b * kABytes + r * 128), r);
            } else if constexpr (FMT == T2C_Q6_K) {
                const int slot = p.q6_grouped ? (r & 7) * 16 + (r >> 3) : r;
                const int off = p.q6_grouped ? RF::goff_of(sb0 + sb, r & 7, p.row_bytes) : RF::off_of(sb0 + sb);
                dequant_q6k_half(smem_u32(raw_ptr + (sb & 1) * kRawBytes + slot * RF::kRow) + off, q, hf,
                                 a_base + static_cast<uint32_t>(b * kABytes + r * 128), r);
            } else {
            dequant_half(raw_ptr + (sb & 1) * kRawBytes + r * 144, q, hf,
                         a_base + static_cast<uint32_t>(b * kABytes + r * 128), r);
            }
            if (FMT == T2C_Q4_K && swiglu)
                dequant_half(rawup_ptr + (sb & 1) * kRawBytes + r * 144, q, hf,
                             aup_base + static_cast<uint32_t>(b * kABytes + r * 128), r);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&a_full[b]);
                if (q == 3) mbar_arrive(&raw_empty[sb & 1]);
            }
        }
    }
    __syncthreads();
    bool ok = !failed;
    if (ok && nch > 0) ok = mbar_wait(&mma_done[(nch - 1) % kNB], static_cast<uint32_t>(((nch - 1) / kNB) & 1));
    if (!ok && tid == 0) report_device_error(T2C_ETIMEOUT);
    if (warp < kDeqWarps) {
        // TMEM lane quadrant of warp w: weight rows 32 (w % 4) ..; warps 0..3 / 4..7 split the columns
        const int quad = warp & 3;
        const int64_t n = n0 + 32 * quad + lane;
        const uint32_t lane_addr = tmem + (static_cast<uint32_t>(32 * quad) << 16);
        const bool split_cols = (mt % 32) == 0;
        const int c_begin = split_cols ? (warp >> 2) * (mt / 2) : 0;
        const int c_end = split_cols ? c_begin + mt / 2 : (warp < 4 ? mt : 0);
        if (p.ksplit > 1 || stacked) {
            // cluster split-K (and the stacked SwiGLU tile, whose gate and up rows sit in
            // different warps' TMEM lanes): every CTA parks its fp32 partials column-major in
            // its own shared memory (reusing the operand buffers and raw stages: every copy has
            // landed and every MMA has completed); the finishing pass below reads them back
            float *red = reinterpret_cast<float *>(smem);
            const int row = 32 * quad + lane;
            if (ok) {
                tc_fence_after();
                for (int c = c_begin; c < c_end; c += 16) {
                    uint32_t v[16];
                    tmem_ld16(lane_addr + static_cast<uint32_t>(c), v);
#pragma unroll
                    for (int j = 0; j < 16; ++j) red[(c + j) * kRowsT + row] = __uint_as_float(v[j]);
                    if (swiglu) {
                        tmem_ld16(lane_addr + static_cast<uint32_t>(mt + c), v);
#pragma unroll
                        for (int j = 0; j < 16; ++j) red[(mt + c + j) * kRowsT + row] = __uint_as_float(v[j]);
                    }
                }
            } else {
                for (int c = c_begin; c < c_end; ++c) {
                    red[c * kRowsT + row] = 0.0f;
                    if (swiglu) red[(mt + c) * kRowsT + row] = 0.0f;
                }
            }
        } else if (ok) {
            tc_fence_after();
            for (int c = c_begin; c < c_end; c += 16) {
                uint32_t g[16], u[16];
                tmem_ld16(lane_addr + static_cast<uint32_t>(c), g);
                if (swiglu) tmem_ld16(lane_addr + static_cast<uint32_t>(mt + c), u);
                if (p.ps != nullptr) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) argmax4_store(p, m0 + c + j, n, N, __uint_as_float(g[j]), true);
                    continue;
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int64_t m = m0 + c + j;
                    if (m < p.M && n < N) {
                        const int64_t o = m * N + n;
                        float v = __uint_as_float(g[j]);
                        if (swiglu) {
                            v = v / (1.0f + __expf(-v)) * __uint_as_float(u[j]);
                        } else {
                            if (p.bias != nullptr) v += p.bias[n];
                            if (p.act) v = gelu_erf_g(v);
                            if (res != nullptr) v += __half2float(res[o]);
                        }
                        if (youtf != nullptr)
                            youtf[o] = v;
                        else
                            yout[o] = __float2half_rn(v);
                    }
                }
            }
        }
    }
    if (p.ksplit > 1 || stacked) {
        const int ks = p.ksplit;
        if (ks > 1)
            asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
        else
            __syncthreads();
        // every CTA of the cluster finishes mt / ks of the columns: per item, one column and four
        // consecutive rows, read as one 16-byte load from each rank's parked partials and summed in
        // rank order (the same order for every column, so the result does not depend on timing)
        const uint32_t red = smem_u32(smem);
        uint32_t rbase[8];
#pragma unroll
        for (int rk = 0; rk < 8; ++rk) {
            rbase[rk] = red;
            if (ks > 1 && rk < ks)
                asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rbase[rk]) : "r"(red), "r"(rk));
        }
        const int cpr = mt / ks, cb = kpart * cpr;
        const int nq = stacked ? kRowsT / 8 : kRowsT / 4;  // row quads finished per column
        // second operand of an item: the up column (SwiGLU) or the up rows 64 below (stacked)
        const uint32_t uoff = swiglu ? static_cast<uint32_t>(mt * kRowsT * 4) : stacked ? (kRowsT / 2) * 4u : 0u;
        for (int it = tid; it < cpr * nq; it += kThreadsG) {
            const int c = cb + it / nq, r = 4 * (it % nq);
            const int64_t m = m0 + c, n = n0 + r;
            float rv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (res != nullptr && !swiglu && !stacked && m < p.M) {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (n + j < N) rv[j] = __half2float(res[m * N + n + j]);
            }
            const uint32_t off = static_cast<uint32_t>((c * kRowsT + r) * 4);
            float g[4], u[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            sum_parked(rbase, ks, off, g);
            if (uoff) sum_parked(rbase, ks, off + uoff, u);
            if (p.ps != nullptr) {
                // best (value, row) of the four rows n .. n + 3; ties keep the lower row
                float best = (n < N && ok) ? g[0] : -INFINITY;
                uint32_t tok = static_cast<uint32_t>(n);
#pragma unroll
                for (int j = 1; j < 4; ++j) {
                    const float v = (n + j < N && ok) ? g[j] : -INFINITY;
                    if (v > best) {
                        best = v;
                        tok = static_cast<uint32_t>(n + j);
                    }
                }
                if (n < N && m < p.M) {
                    p.ps[m * p.G + (n >> 2)] = best;
                    p.pt[m * p.G + (n >> 2)] = tok;
                }
                continue;
            }
            if (!ok || m >= p.M) continue;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (n + j >= N) continue;
                const int64_t o = m * N + n + j;
                float v = g[j];
                if (swiglu || stacked) {
                    v = v / (1.0f + __expf(-v)) * u[j];
                } else {
                    if (p.bias != nullptr) v += p.bias[n + j];
                    if (p.act) v = gelu_erf_g(v);
                    if (res != nullptr) v += rv[j];
                }
                if (youtf != nullptr)
                    youtf[o] = v;
                else
                    yout[o] = __float2half_rn(v);
            }
        }
        // partners keep their shared memory until every CTA of the cluster has read it
        if (ks > 1)
            asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(static_cast<uint32_t>(p.tmem_cols))
                     : "memory");
}

PFN_cuTensorMapEncodeTiled tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled encode = [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            fn = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled>(fn);
    }();
    return encode;
}

// rows_per_box kRowsT: one TMA row per weight row; 16: rows are eight-row groups (grouped Q6_K)
bool encode_raw(CUtensorMap *map, const uint8_t *w, int64_t n, int64_t row_bytes, int box_words,
                int rows_per_box = kRowsT) {
    const auto enc = tensor_map_encoder();
    if (!enc || row_bytes % 16 || reinterpret_cast<uintptr_t>(w) % 16) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes / 4), static_cast<cuuint64_t>(n)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_words), static_cast<cuuint32_t>(rows_per_box)};
    const cuuint32_t es[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint8_t *>(w), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_x(CUtensorMap *map, const __half *x, int64_t m, int64_t k, int mt) {
    const auto enc = tensor_map_encoder();
    if (!enc || reinterpret_cast<uintptr_t>(x) % 16 || (k * 2) % 16) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(m)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(k * 2)};
    const cuuint32_t box[2] = {kKC, static_cast<cuuint32_t>(mt)};
    const cuuint32_t es[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(x), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

int qgemm(const QGemmArgs &a, cudaStream_t stream) {
    if (a.M <= 4 || a.K % 256 || a.K > 65536 || a.M > INT32_MAX || a.nw < 1 || a.nw > 3 || (a.w_up && a.nw != 1))
        return T2C_EUNSUPPORTED;
    if (a.fmt != T2C_Q4_K && a.fmt != T2C_Q6_K && a.fmt != T2C_Q8_0) return T2C_EUNSUPPORTED;
    if (a.fmt != T2C_Q4_K && a.w_up) return T2C_EUNSUPPORTED;
    if (a.ps && (a.nw != 1 || a.w_up || !a.pt)) return T2C_EUNSUPPORTED;
    if ((a.bias || a.act) && (a.nw != 1 || a.w_up || a.ps)) return T2C_EUNSUPPORTED;
    for (int i = 0; i < a.nw; ++i)
        if (a.N[i] <= 0 || a.N[i] > INT32_MAX) return T2C_EUNSUPPORTED;
    GemmParams p = {};
    p.swiglu = a.w_up != nullptr;
    const int cap = p.swiglu ? 128 : 256;
    int64_t mt = (a.M + 15) / 16 * 16;
    if (mt > cap) mt = cap;
    p.mt = static_cast<int>(mt);
    // SwiGLU at up to 32 tokens: 64 gate rows over the same 64 up rows fill one 128-row tile, so the
    // CTA needs the plain linear's shared memory (two CTAs per SM) and the grid twice the tiles
    if (p.swiglu && mt <= 32) {
        p.swiglu = 0;
        p.stacked = 1;
    }
    const int rows_t = p.stacked ? kRowsT / 2 : kRowsT;
    const int64_t row_bytes = a.K / 256 * (a.fmt == T2C_Q6_K ? 210 : a.fmt == T2C_Q8_0 ? 272 : 144);
    const int box = a.fmt == T2C_Q6_K ? 56 : a.fmt == T2C_Q8_0 ? 68 : 36;
    const size_t raw_bytes = static_cast<size_t>(kRowsT) * (a.fmt == T2C_Q6_K ? 224 : a.fmt == T2C_Q8_0 ? 272 : 144);
    p.nw = a.nw;
    p.q6_grouped = a.fmt == T2C_Q6_K && row_bytes % 16 != 0;
    p.row_bytes = static_cast<int>(row_bytes);
    if (p.q6_grouped)
        for (int i = 0; i < a.nw; ++i)
            if (a.N[i] % 8) return T2C_EUNSUPPORTED;
    int64_t row_tiles = 0;
    for (int i = 0; i < a.nw; ++i) {
        const bool ok = p.q6_grouped ? encode_raw(&p.wmap[i], a.w[i], a.N[i] / 8, 8 * row_bytes, box, kRowsT / 8)
                                     : encode_raw(&p.wmap[i], a.w[i], a.N[i], row_bytes, box, rows_t);
        if (!ok) return T2C_EUNSUPPORTED;
        p.tile0[i] = static_cast<int>(row_tiles);
        row_tiles += (a.N[i] + rows_t - 1) / rows_t;
        p.Nw[i] = a.N[i];
        p.y[i] = a.y[i];
        p.yf[i] = a.yf[i];
        p.res[i] = a.res[i];
    }
    p.tile0[a.nw] = static_cast<int>(row_tiles);
    if ((p.swiglu || p.stacked) && !encode_raw(&p.umap, a.w_up, a.N[0], row_bytes, box, rows_t))
        return T2C_EUNSUPPORTED;
    p.ps = a.ps;
    p.pt = a.pt;
    p.G = a.G;
    p.bias = a.bias;
    p.act = a.act;
    if (!encode_x(&p.xmap, a.x, a.M, a.K, p.mt)) return T2C_EUNSUPPORTED;
    // split K over a cluster when there are too few (row tile, token tile) pairs to fill the GPU
    const int64_t tiles = row_tiles * ((a.M + p.mt - 1) / p.mt);
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    p.ksplit = 1;
    const int nsb_all = static_cast<int>(a.K / 256);
    if (p.mt <= (p.swiglu ? 32 : 64)) {
        while (p.ksplit < 8 && tiles * p.ksplit < sms && nsb_all % (p.ksplit * 2) == 0 && nsb_all / (p.ksplit * 2) >= 2)
            p.ksplit *= 2;
    } else {
        // larger token tiles: split only while the doubled grid still fits on the SMs, and only where
        // the parked fp32 partials (mt columns x 128 rows, x 2 with SwiGLU) fit in the operand buffers
        // and raw stages they reuse once the main loop is over
        const size_t red = static_cast<size_t>(p.swiglu ? 2 : 1) * p.mt * kRowsT * 4;
        const size_t reusable = static_cast<size_t>(kNB) * kABytes * (p.swiglu ? 2 : 1) +
                                static_cast<size_t>(kNB) * p.mt * 128 + 2 * raw_bytes * (p.swiglu ? 2 : 1);
        // (each CTA keeps at least 12 super-blocks: with fewer the DSMEM sum of 128 x mt partials
        // costs more than the split gains; measured at K = 4096 vs 12288, M = 256)
        while (red <= reusable && p.ksplit < 8 && tiles * p.ksplit * 2 <= sms && nsb_all % (p.ksplit * 2) == 0 &&
               nsb_all / (p.ksplit * 2) >= 12)
            p.ksplit *= 2;
    }
    p.M = a.M;
    p.K = static_cast<int>(a.K);
    int cols = 32;
    while (cols < (p.swiglu ? 2 : 1) * p.mt) cols *= 2;
    p.tmem_cols = cols;
    const size_t smem = 1024 + static_cast<size_t>(kNB) * kABytes * (p.swiglu ? 2 : 1) +
                        static_cast<size_t>(kNB) * p.mt * 128 + 2 * raw_bytes * (p.swiglu ? 2 : 1) +
                        (4 + 3 * kNB) * 8 + 16;
    constexpr size_t kLimit = 226 * 1024;  // dynamic bytes; the kernel's static words sit beside them
    if (smem > kLimit) return T2C_EUNSUPPORTED;
    static bool configured[3][64] = {};
    int device = 0;
    cudaGetDevice(&device);
    const int slot = device < 0 ? 0 : (device > 63 ? 63 : device);
    const int fi = a.fmt == T2C_Q6_K ? 1 : a.fmt == T2C_Q8_0 ? 2 : 0;
    if (!configured[fi][slot]) {
        const cudaError_t e =
            fi == 1 ? cudaFuncSetAttribute(qgemm_kernel<T2C_Q6_K>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(kLimit))
            : fi == 2 ? cudaFuncSetAttribute(qgemm_kernel<T2C_Q8_0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kLimit))
                      : cudaFuncSetAttribute(qgemm_kernel<T2C_Q4_K>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kLimit));
        if (e != cudaSuccess) return set_error(T2C_ECUDA, "qgemm: cudaFuncSetAttribute failed");
        configured[fi][slot] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(row_tiles * p.ksplit),
                       static_cast<unsigned>((a.M + p.mt - 1) / p.mt));
    cfg.blockDim = dim3(kThreadsG);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = static_cast<unsigned>(p.ksplit);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const cudaError_t err = fi == 1   ? cudaLaunchKernelEx(&cfg, qgemm_kernel<T2C_Q6_K>, p)
                            : fi == 2 ? cudaLaunchKernelEx(&cfg, qgemm_kernel<T2C_Q8_0>, p)
                                      : cudaLaunchKernelEx(&cfg, qgemm_kernel<T2C_Q4_K>, p);
    if (err != cudaSuccess) return set_error(T2C_ECUDA, "qgemm launch: %s", cudaGetErrorString(err));
    return T2C_OK;
}

cudaError_t status_qgemm(unsigned int *bits, int clear, cudaStream_t s) { return read_tu_status(bits, clear, s); }

}  // namespace t2c
