// Causal GQA prefill attention on tcgen05 tensor cores (D = 128), the B200
// form of the reference's sdpa_causal_f32 / llama_flash_attn programs
// (src/models/quantized_qwen3/shaders/sdpa_causal_f32.py:22-142).
//
// CTA = one warpgroup (128 threads) on (sequence b, head h, 128-query tile);
// thread r owns query row r of the tile, which is TMEM lane r.  Per 128-key
// tile j of 64 cache rows up to positions[b] + (last query of the tile):
//   S = Q K_j^T   tcgen05.mma kind::f16, M = 128 queries, N = 64 keys,
//                 K = D in 8 steps, fp32 accumulators in TMEM columns 0..63;
//   online softmax per row in fp32 (log2 domain) from tcgen05.ld of S, P = fp16
//                 exp2(s - m) written to shared memory as the next A operand;
//                 when a row's maximum moves, its O row in TMEM is rescaled
//                 (tcgen05.ld / st);
//   O += P V_j    M = 128, N = D (V read MN-major), K = 64 keys in 4 steps,
//                 TMEM columns 128..255.
// Q, K, V and P tiles sit in shared memory in the 128-byte-swizzled layout the
// UMMA descriptors name ([chunks of 64 values][rows][128 B], 16-byte unit u of
// row r at ((u ^ r) mod 8)); K / V tiles are double-buffered with cp.async
// (rows past the cache zero-filled).  112 KB of shared memory and 256 TMEM
// columns per CTA: two CTAs per SM, so one's softmax overlaps the other's MMAs.  One thread issues the MMAs; a
// commit per tile signals S (and with it every earlier MMA) to the warpgroup
// through an mbarrier whose waits are bounded.
#include <float.h>

#include "common.cuh"

namespace t2c {
namespace {

constexpr int kUQ = 128;                 // queries per CTA (UMMA M, TMEM lanes)
constexpr int kUK = 64;                  // keys per tile (UMMA N of S, K of P V)
constexpr int kUQTile = kUQ * 128 * 2;   // Q: 128 rows x 128 values, two 64-value chunks of 16 KB
constexpr int kUKTile = kUK * 128 * 2;   // K or V: 64 rows x 128 values, two chunks of 8 KB
constexpr int kUPTile = kUQ * kUK * 2;   // P: 128 rows x 64 keys, one chunk
// Q, K x 2, V x 2, P, barrier + TMEM slot: 112 KB + 64 B, so two CTAs share an SM (the kernel checks
// that the dynamic shared window starts on the 1024-byte boundary the swizzle atoms need)
constexpr int kUSmem = kUQTile + 4 * kUKTile + kUPTile + 64;

// 16-byte unit u (0..15) of row r in a tile of two 64-value chunks `chunk` bytes apart, 128-byte swizzle
__device__ __forceinline__ uint32_t sw_off(int r, int u, int chunk) {
    return static_cast<uint32_t>((u >> 3) * chunk + r * 128 + (((u & 7) ^ (r & 7)) << 4));
}

// K-major operand, 128-byte swizzle: 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t desc_k(uint32_t saddr) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1u) << 16) |
           (static_cast<uint64_t>(1024u >> 4) << 32) | (static_cast<uint64_t>(1u) << 46) |
           (static_cast<uint64_t>(2u) << 61);
}

// MN-major operand, 128-byte swizzle: 64-value atoms along N one V chunk (8 KB) apart (leading), 8-row
// K groups 1024 B apart (stride).
__device__ __forceinline__ uint64_t desc_mn(uint32_t saddr) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(uint32_t(kUKTile / 2) >> 4) << 16) |
           (static_cast<uint64_t>(1024u >> 4) << 32) | (static_cast<uint64_t>(1u) << 46) |
           (static_cast<uint64_t>(2u) << 61);
}

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, bool acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc ? 1u : 0u)
        : "memory");
}

__device__ __forceinline__ void commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void ld16(uint32_t taddr, uint32_t v[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 consecutive columns of this thread's lane; the caller waits (tcgen05.wait::ld) before use.
__device__ __forceinline__ void ld32_nowait(uint32_t taddr, uint32_t *v) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
        "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}

__device__ __forceinline__ void st16(uint32_t taddr, const uint32_t v[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

__device__ __forceinline__ void cp16(uint32_t dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// MASKED: keys [0, S) under an additive fp16 mask (sequence b's element (t, key) at mask + b * m_sb +
// t * m_st + key; values <= -FLT_MAX / 2 hide the key) instead of the causal rule.  F32IO: fp32 q and
// output (rounded to fp16 for the tensor cores on the way in).
template <bool MASKED, bool F32IO>
__global__ void __launch_bounds__(128, 2) attn_prefill_umma_kernel(
    const void *__restrict__ qv, const __half *__restrict__ kc, const __half *__restrict__ vc,
    void *__restrict__ outv, const int32_t *__restrict__ positions, int T, int NH, int NK, int64_t cb, int64_t cs,
    int64_t ch, int64_t q_sb, int64_t q_st, int64_t q_sh, int64_t o_sb, int64_t o_st, int64_t o_sh,
    float scale_log2, const __half *__restrict__ mask, int64_t m_sb, int64_t m_st, int S) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t qs = smem_u32(smem);
    const uint32_t ks0 = qs + kUQTile, vs0 = ks0 + 2 * kUKTile, ps = vs0 + 2 * kUKTile;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + kUQTile + 4 * kUKTile + kUPTile);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar + 2);
    if (qs & 1023u) {  // swizzle atoms need 1024-byte alignment: report, compute nothing
        if (threadIdx.x == 0) report_device_error(T2C_EUNSUPPORTED);
        return;
    }
    const int tid = threadIdx.x, warp = tid >> 5;
    const int qtiles = (T + kUQ - 1) / kUQ;
    const int qt = qtiles - 1 - static_cast<int>(blockIdx.x % qtiles);  // heaviest tiles first
    const int h = (blockIdx.x / qtiles) % NH;
    const int b = blockIdx.x / (qtiles * NH);
    const int kh = h / (NH / NK);
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(256u)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(tmem_slot);
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * warp) << 16);
    pdl_wait();
    pdl_trigger();

    const int base = MASKED ? 0 : positions[b];
    const int q0 = qt * kUQ;
    const int last_key = MASKED ? S - 1 : base + min(T - 1, q0 + kUQ - 1);
    const int ntiles = last_key / kUK + 1;
    const int row = tid;
    const int qpos = base + q0 + row;  // keys <= qpos are visible to this row
    const __half *kbase = kc + b * cb + kh * ch;
    const __half *vbase = vc + b * cb + kh * ch;

    // Q row -> swizzled tile (rows past T are zero)
    {
        const int tq = q0 + row;
        const int64_t qoff = b * q_sb + static_cast<int64_t>(tq) * q_st + h * q_sh;
#pragma unroll
        for (int u = 0; u < 16; ++u) {
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (tq < T) {
                if constexpr (F32IO) {
                    const float4 a = reinterpret_cast<const float4 *>(static_cast<const float *>(qv) + qoff)[2 * u];
                    const float4 c = reinterpret_cast<const float4 *>(static_cast<const float *>(qv) + qoff)[2 * u + 1];
                    v = make_uint4(pack2(a.x, a.y), pack2(a.z, a.w), pack2(c.x, c.y), pack2(c.z, c.w));
                } else {
                    v = reinterpret_cast<const uint4 *>(static_cast<const __half *>(qv) + qoff)[u];
                }
            }
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(qs + sw_off(row, u, kUQTile / 2)), "r"(v.x), "r"(v.y),
                         "r"(v.z), "r"(v.w)
                         : "memory");
        }
    }
    // key / value tile j into buffer j & 1: threads 0..63 copy key rows j * 64 + r of K, 64..127 those of V
    auto load_kv = [&](int j) {
        const int r = row & (kUK - 1);
        const int key = j * kUK + r;
        const bool in = key <= last_key;
        const int64_t off = in ? static_cast<int64_t>(key) * cs : 0;
        const uint32_t dst = (row < kUK ? ks0 : vs0) + (j & 1) * kUKTile;
        const __half *src = (row < kUK ? kbase : vbase) + off;
#pragma unroll
        for (int u = 0; u < 16; ++u) cp16(dst + sw_off(r, u, kUKTile / 2), src + 8 * u, in ? 16u : 0u);
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    load_kv(0);

    const uint32_t idesc_s = (1u << 4) | (static_cast<uint32_t>(kUK >> 3) << 17) | (static_cast<uint32_t>(kUQ >> 4) << 24);
    // P V: N = D = 128, B = V read MN-major
    const uint32_t idesc_o = (1u << 4) | (1u << 16) | (128u >> 3 << 17) | (static_cast<uint32_t>(kUQ >> 4) << 24);
    float m_run = -FLT_MAX, l_run = 0.0f;
    bool failed = false;
    int issued = 0;  // commits so far (uniform over the CTA)
    for (int j = 0; j < ntiles; ++j) {
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        const uint32_t kt = ks0 + (j & 1) * kUKTile, vt = vs0 + (j & 1) * kUKTile;
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
            for (int s = 0; s < 8; ++s) {
                const uint32_t qo = static_cast<uint32_t>((s >> 2) * (kUQTile / 2) + 32 * (s & 3));
                const uint32_t ko = static_cast<uint32_t>((s >> 2) * (kUKTile / 2) + 32 * (s & 3));
                umma(tmem, desc_k(qs + qo), desc_k(kt + ko), idesc_s, s > 0);
            }
            commit(bar);
        }
        ++issued;
        // a wait that runs out stops the whole CTA at the same point (one vote, every thread)
        const bool ok = mbar_wait(bar, static_cast<uint32_t>(j & 1));
        if (__syncthreads_or(!ok)) {
            failed = true;
            break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        // every MMA issued so far is complete: the other buffer (tile j - 1) is free
        if (j + 1 < ntiles) load_kv(j + 1);
        const int k0 = j * kUK;
        const bool diag = k0 + kUK - 1 > base + q0;  // some key of the tile is past some query of the CTA
        // the whole S row (64 fp32) in registers: two loads, one wait
        uint32_t sv[kUK];
#pragma unroll
        for (int c = 0; c < kUK / 32; ++c) ld32_nowait(lane_base + static_cast<uint32_t>(32 * c), sv + 32 * c);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        float mx = -FLT_MAX;
        if constexpr (MASKED) {
            // this row's 64 mask values of the tile (the last real query row for padding rows)
            const __half *mrow = mask + b * m_sb + static_cast<int64_t>(min(q0 + row, T - 1)) * m_st;
#pragma unroll
            for (int i = 0; i < kUK; ++i) {
                const int key = k0 + i;
                const float mv = key < S ? __half2float(mrow[key]) : -FLT_MAX;
                const bool vis = mv > -1.7014117e38f;
                const float x = fmaf(mv, 1.4426950408889634f, __uint_as_float(sv[i]) * scale_log2);
                sv[i] = __float_as_uint(vis ? x : -FLT_MAX);
                mx = fmaxf(mx, vis ? x : -FLT_MAX);
            }
        } else {
#pragma unroll
            for (int i = 0; i < kUK; ++i) {
                const float x = __uint_as_float(sv[i]) * scale_log2;
                const bool vis = !diag || k0 + i <= qpos;
                sv[i] = __float_as_uint(vis ? x : -FLT_MAX);
                mx = fmaxf(mx, vis ? x : -FLT_MAX);
            }
        }
        // The running maximum moves only when a score exceeds it by more than 8 (log2 units): P stays below
        // 2^8 (exact enough in fp16, far from its range), O is rescaled rarely, and O / l is the same for any
        // common reference point.  A row with nothing visible yet keeps m = -FLT_MAX and l = 0.
        const float m_new = (m_run == -FLT_MAX || mx > m_run + 8.0f) ? fmaxf(m_run, mx) : m_run;
        const float corr = m_run == -FLT_MAX ? 0.0f : exp2f(m_run - m_new);
        float lsum = 0.0f;
#pragma unroll
        for (int c = 0; c < kUK / 16; ++c) {
            float p[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float x = __uint_as_float(sv[16 * c + i]);
                p[i] = x == -FLT_MAX ? 0.0f : exp2f(x - m_new);
                lsum += p[i];
            }
            // keys 16c .. 16c + 15 = 16-byte units 2c, 2c + 1 of row `row` (one 64-key chunk)
            const uint32_t d0 = ps + sw_off(row, 2 * c, kUPTile), d1 = ps + sw_off(row, 2 * c + 1, kUPTile);
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(d0), "r"(pack2(p[0], p[1])),
                         "r"(pack2(p[2], p[3])), "r"(pack2(p[4], p[5])), "r"(pack2(p[6], p[7]))
                         : "memory");
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(d1), "r"(pack2(p[8], p[9])),
                         "r"(pack2(p[10], p[11])), "r"(pack2(p[12], p[13])), "r"(pack2(p[14], p[15]))
                         : "memory");
        }
        l_run = l_run * corr + lsum;
        // tcgen05.ld / st are warp-collective: the warp rescales its 32 rows of O together when any row's
        // maximum moved (the others multiply by 1); the P V of tile j - 1 has completed
        if (j > 0 && __any_sync(0xffffffffu, corr != 1.0f)) {
#pragma unroll 1
            for (int c = 0; c < 8; ++c) {
                uint32_t v[16];
                ld16(lane_base + 128u + static_cast<uint32_t>(16 * c), v);
#pragma unroll
                for (int i = 0; i < 16; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * corr);
                st16(lane_base + 128u + static_cast<uint32_t>(16 * c), v);
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        }
        m_run = m_new;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
            for (int s = 0; s < kUK / 16; ++s)
                umma(tmem + 128u, desc_k(ps + static_cast<uint32_t>(32 * s)), desc_mn(vt + static_cast<uint32_t>(2048 * s)),
                     idesc_o, j > 0 || s > 0);
        }
    }
    // the last P V (or, after a timeout, whatever is in flight) before O is read and TMEM is freed
    __syncthreads();
    if (tid == 0) commit(bar);
    const bool done = __syncthreads_and(mbar_wait(bar, static_cast<uint32_t>(issued & 1)));
    if (failed || !done) {
        if (tid == 0) report_device_error(T2C_ETIMEOUT);
    } else {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int tq = q0 + row;
        const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
        const int64_t ooff = b * o_sb + static_cast<int64_t>(tq) * o_st + h * o_sh;
        uint4 *dst = reinterpret_cast<uint4 *>(static_cast<__half *>(outv) + ooff);
        float4 *dstf = reinterpret_cast<float4 *>(static_cast<float *>(outv) + ooff);
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
            uint32_t v[16];
            ld16(lane_base + 128u + static_cast<uint32_t>(16 * c), v);
            if (F32IO && tq < T) {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    dstf[4 * c + i] = make_float4(__uint_as_float(v[4 * i]) * inv, __uint_as_float(v[4 * i + 1]) * inv,
                                                  __uint_as_float(v[4 * i + 2]) * inv,
                                                  __uint_as_float(v[4 * i + 3]) * inv);
            } else if (tq < T) {
                const float f[16] = {__uint_as_float(v[0]),  __uint_as_float(v[1]),  __uint_as_float(v[2]),
                                     __uint_as_float(v[3]),  __uint_as_float(v[4]),  __uint_as_float(v[5]),
                                     __uint_as_float(v[6]),  __uint_as_float(v[7]),  __uint_as_float(v[8]),
                                     __uint_as_float(v[9]),  __uint_as_float(v[10]), __uint_as_float(v[11]),
                                     __uint_as_float(v[12]), __uint_as_float(v[13]), __uint_as_float(v[14]),
                                     __uint_as_float(v[15])};
                dst[2 * c] = make_uint4(pack2(f[0] * inv, f[1] * inv), pack2(f[2] * inv, f[3] * inv),
                                        pack2(f[4] * inv, f[5] * inv), pack2(f[6] * inv, f[7] * inv));
                dst[2 * c + 1] = make_uint4(pack2(f[8] * inv, f[9] * inv), pack2(f[10] * inv, f[11] * inv),
                                            pack2(f[12] * inv, f[13] * inv), pack2(f[14] * inv, f[15] * inv));
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256u) : "memory");
}

}  // namespace

// Launches the tcgen05 prefill attention for D = 128 (causal from positions[b], or with an additive
// mask when `mask` is given: keys [0, S)); T2C_EUNSUPPORTED when the strides or alignment do not suit it
// (the caller then takes the mma.sync kernel).
int attn_prefill_umma(const void *q, const void *k_cache, const void *v_cache, void *out, const int32_t *positions,
                      int64_t B, int64_t T, int64_t NH, int64_t NK, int64_t cb, int64_t cs, int64_t ch, int64_t qb,
                      int64_t qt, int64_t qh, int64_t ob, int64_t ot, int64_t oh, float scale, cudaStream_t stream,
                      const void *mask, int64_t m_sb, int64_t m_st, int64_t S, bool f32io) {
    const auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    const int64_t qa = f32io ? 4 : 8;  // elements per 16 bytes of q / out
    if (!al16(q) || !al16(k_cache) || !al16(v_cache) || !al16(out) || qb % qa || qt % qa || qh % qa || ob % qa ||
        ot % qa || oh % qa || cb % 8 || cs % 8 || ch % 8)
        return T2C_EUNSUPPORTED;
    if (mask == nullptr && (positions == nullptr || f32io)) return T2C_EUNSUPPORTED;
    static bool configured[4][64] = {};
    int device = 0;
    cudaGetDevice(&device);
    const int slot = device < 0 ? 0 : (device > 63 ? 63 : device);
    const int variant = (mask != nullptr ? 2 : 0) + (f32io ? 1 : 0);
    void (*kern)(const void *, const __half *, const __half *, void *, const int32_t *, int, int, int, int64_t,
                 int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, float, const __half *, int64_t,
                 int64_t, int) = variant == 0   ? attn_prefill_umma_kernel<false, false>
                                 : variant == 2 ? attn_prefill_umma_kernel<true, false>
                                 : variant == 3 ? attn_prefill_umma_kernel<true, true>
                                                : nullptr;
    if (kern == nullptr) return T2C_EUNSUPPORTED;
    if (!configured[variant][slot]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kUSmem) != cudaSuccess)
            return set_error(T2C_ECUDA, "attn_prefill: cudaFuncSetAttribute failed");
        configured[variant][slot] = true;
    }
    const int64_t tiles = (T + kUQ - 1) / kUQ;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(B * NH * tiles));
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = kUSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t err = cudaLaunchKernelEx(
        &cfg, kern, q, static_cast<const __half *>(k_cache), static_cast<const __half *>(v_cache), out, positions,
        static_cast<int>(T), static_cast<int>(NH), static_cast<int>(NK), cb, cs, ch, qb, qt, qh, ob, ot, oh,
        1.4426950408889634f * scale, static_cast<const __half *>(mask), m_sb, m_st, static_cast<int>(S));
    if (err != cudaSuccess) return set_error(T2C_ECUDA, "attn_prefill (tcgen05) launch: %s", cudaGetErrorString(err));
    return T2C_OK;
}

cudaError_t status_attn_tc(unsigned int *bits, int clear, cudaStream_t s) { return read_tu_status(bits, clear, s); }

}  // namespace t2c
