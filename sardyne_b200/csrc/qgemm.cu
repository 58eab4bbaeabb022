// Prefill GEMM for Q4_K / Q6_K weights on the 5th-generation tensor cores: y[t][r] = W[r] . x[t]
// for many tokens, bit-identical to the reference's per-block integer dot products (reference
// csrc/quant.c:176-235 and the combine of quant.h:84-91), which the matvec reproduces too.
//
// Exactness. Per 256-element superblock b the reference forms integer sums and rounds one float
// term per (row, token, b), added to the row's total in block order. The integer sums become
// int8 MMAs (tcgen05.mma kind::i8, int32 accumulators in TMEM):
//   Q4_K  isum = sum_e sc(e) q(e) y(e) with sc*q <= 945 split as 32*hi + lo (hi <= 29, lo <= 31),
//         msum = sum_e m(e) y(e) with the 6-bit min of e's sub-block repeated over its 32 lanes;
//   Q6_K  isum = sum_e sc(e) (q(e) - 32) y(e), the product in [-4064, 4096] split as 64*hi + lo
//         (hi in [-64, 64], lo in [0, 63]).
// So the A operand of a tile is the expanded weight products (two or three int8 planes), B the
// Q8_K activations; every K step of 32 is one MMA per plane into that plane's accumulator. After a
// superblock's 8 K steps the epilogue reads the accumulators (tcgen05.ld), rebuilds isum/msum and
// applies the reference's float combine, keeping each (row, token) total in registers.
//
// Tile: 128 weight rows (MMA M) x 128 tokens (MMA N), 256 threads. Operands sit in shared memory
// in the no-swizzle K-major core-matrix layout: byte (row, k) of a plane at
// (k / 16) * (rows * 16) + row * 16 + k % 16, i.e. 8-row x 16-byte core matrices, 128 B apart
// along M and rows*16 B apart along K. The next superblock's raw slabs, B tile and token scales
// are requested with cp.async before the current superblock's MMAs are issued, so their latency
// overlaps the MMAs and the epilogue; expansion, MMA and epilogue of one superblock still follow
// each other.
//
// Split along K. A product of few tiles (a 2048-row matrix at a few hundred tokens: 16-86 CTAs on
// 148 SMs) gives each CTA of grid.z a range of superblocks; instead of adding its terms to
// registers the epilogue stores them, terms[b][token][row], and qgemm_reduce_kernel adds each
// output's terms in superblock order from zero, exactly the sum the single CTA forms.
//
// The 32-element formats (Q8_0, Q4_0, Q5_0; reference csrc/quant.c:148-189) go through
// qgemm32_kernel: per block the reference forms the integer sum s of its 32 products and adds
// (float)s * (dw * dx) to the row's total in block order (quant.c:160). A block's weight values
// with the bias removed (Q8_0 as stored, Q4_0 q - 8, Q5_0 q - 16) are int8, so one MMA of K = 32
// gives s for the whole 128 x 128 tile; KB = 4 blocks per step go to their own accumulators
// (4 x 128 TMEM columns) and the epilogue adds the 4 terms per (row, token) in block order. Q8_0
// needs no expansion beyond the copy into the core-matrix layout (the slab's 16-byte chunks of
// 8 rows are already 8-row core matrices).
#include "common.cuh"

#include <string.h>

#include <mutex>

namespace sdy {
namespace {

constexpr int GM = 128;           // weight rows per tile
constexpr int GN = GEMM_TILE_TOKENS;  // tokens per tile
constexpr int G_THREADS = 256;
constexpr int PLANE = GM * 256;   // bytes of one expanded A plane (one superblock)
constexpr int BTILE = GN * 256;   // bytes of the B tile
constexpr uint32_t TMEM_COLS = 512;
constexpr long long WAIT_LIMIT = 1ll << 22;  // mbarrier polls before giving up (about a second)

__device__ unsigned int g_qgemm_status;  // nonzero: an MMA completion wait timed out

template <int TYPE> struct GemmPlanes { static constexpr int n = TYPE == T_Q4_K ? 3 : 2; };

// Shared memory: the expanded A planes, two B tiles and two yd rows (superblock b+1 arrives by
// cp.async while b is multiplied), d/dmin per row, the raw slabs of the next superblock, mbarrier.
__host__ __device__ constexpr int g_raw_bytes(int type) { return (GM / GROUP_ROWS) * slab_bytes(type); }
__host__ __device__ constexpr int g_smem_bytes(int planes, int type) {
    return planes * PLANE + 2 * BTILE + 2 * GN * 4 + 2 * GM * 4 + g_raw_bytes(type) + 16;
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

// No-swizzle K-major matrix descriptor (version 1): start, LBO = distance of the two 16-byte K
// halves of a 32-byte K step, SBO = distance of consecutive 8-row core matrices.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}

// kind::i8 instruction descriptor: s32 accumulator, s8 A and B, both K-major, M = GM, N = the
// tile's valid tokens rounded up to a multiple of 16 (16 .. GN; the B rows past the valid tokens
// are zero), so a tile of few tokens (an expert's slots in MoE prefill) costs MMAs of its width.
__device__ __forceinline__ uint32_t idesc_i8(int nv) {
    const uint32_t n = (uint32_t)min(GN, max(16, (nv + 15) & ~15));
    return (2u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((uint32_t)(GM >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, int32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}

__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// Bounded wait for phase `parity` of the mbarrier; false when the limit ran out.
__device__ __forceinline__ bool mbar_wait(uint32_t mbar, uint32_t parity) {
    for (long long it = 0; it < WAIT_LIMIT; it++) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(done)
            : "r"(mbar), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

// Byte k of a plane row in the core-matrix layout.
__device__ __forceinline__ int plane_off(int rows, int row, int k) { return (k >> 4) * (rows * 16) + row * 16 + (k & 15); }

// 4 nibbles (one per byte of L, each 0..15) times the scale s (0..63): products split as
// 32*hi + lo, returned as 4 hi bytes and 4 lo bytes.
__device__ __forceinline__ void mul_split32(uint32_t L, uint32_t s, uint32_t &hi, uint32_t &lo) {
    const uint32_t p0 = (L & 0x00FF00FFu) * s, p1 = ((L >> 8) & 0x00FF00FFu) * s;  // 16-bit lanes, <= 945
    hi = ((p0 >> 5) & 0x001F001Fu) | (((p1 >> 5) & 0x001F001Fu) << 8);
    lo = (p0 & 0x001F001Fu) | ((p1 & 0x001F001Fu) << 8);
}

// Expand one (row, superblock) half of the A tile. Q4_K: part p covers the slab's chunks 4p..4p+3
// (elements 128p .. 128p+127), Q6_K: half p of the superblock.
template <int TYPE>
__device__ __forceinline__ void expand_half(const uint8_t *slab, int r8, int row, int part, uint8_t *sa, float *dr,
                                            float *dmr) {
    if constexpr (TYPE == T_Q4_K) {
        const uint4 hdr = *(const uint4 *)(slab + r8 * 16);
        const uint32_t sc0 = hdr.y & 0x3F3F3F3F, m0 = hdr.z & 0x3F3F3F3F;
        const uint32_t sc1 = (hdr.w & 0x0F0F0F0F) | ((hdr.y >> 2) & 0x30303030);
        const uint32_t m1 = ((hdr.w >> 4) & 0x0F0F0F0F) | ((hdr.z >> 2) & 0x30303030);
        if (part == 0) {
            dr[row] = __half2float(__ushort_as_half((uint16_t)(hdr.x & 0xFFFF)));
            dmr[row] = __half2float(__ushort_as_half((uint16_t)(hdr.x >> 16)));
        }
        uint4 q[4];
#pragma unroll
        for (int i = 0; i < 4; i++) q[i] = *(const uint4 *)(slab + 128 + (4 * part + i) * 128 + r8 * 16);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int c = 4 * part + i, j = c >> 1, h = c & 1;  // chunk c: bytes 16h.. of 64-element chunk j
            const uint32_t scw = j < 2 ? sc0 : sc1, mw = j < 2 ? m0 : m1;
            const uint32_t s_lo = (scw >> (16 * (j & 1))) & 0xFF, s_hi = (scw >> (16 * (j & 1) + 8)) & 0xFF;
            const uint32_t m_lo = (mw >> (16 * (j & 1))) & 0xFF, m_hi = (mw >> (16 * (j & 1) + 8)) & 0xFF;
            uint32_t hl[4], ll[4], hh[4], lh[4];
            const uint32_t w[4] = {q[i].x, q[i].y, q[i].z, q[i].w};
#pragma unroll
            for (int k = 0; k < 4; k++) {
                mul_split32(w[k] & 0x0F0F0F0F, s_lo, hl[k], ll[k]);
                mul_split32((w[k] >> 4) & 0x0F0F0F0F, s_hi, hh[k], lh[k]);
            }
            // low nibbles: elements 64j + 16h + 0..15 (sub-block 2j) -> plane 4j + h
            // high nibbles: elements 64j + 32 + 16h + 0..15 (sub-block 2j+1) -> plane 4j + 2 + h
            const int off_l = plane_off(GM, row, 64 * j + 16 * h), off_h = plane_off(GM, row, 64 * j + 32 + 16 * h);
            *(uint4 *)(sa + off_l) = make_uint4(hl[0], hl[1], hl[2], hl[3]);
            *(uint4 *)(sa + PLANE + off_l) = make_uint4(ll[0], ll[1], ll[2], ll[3]);
            *(uint4 *)(sa + off_h) = make_uint4(hh[0], hh[1], hh[2], hh[3]);
            *(uint4 *)(sa + PLANE + off_h) = make_uint4(lh[0], lh[1], lh[2], lh[3]);
            const uint32_t ml = m_lo * 0x01010101u, mh = m_hi * 0x01010101u;
            *(uint4 *)(sa + 2 * PLANE + off_l) = make_uint4(ml, ml, ml, ml);
            *(uint4 *)(sa + 2 * PLANE + off_h) = make_uint4(mh, mh, mh, mh);
        }
    } else {  // Q6_K half `part`: elements 128p .. 128p+127
        const uint4 scv = *(const uint4 *)(slab + 1536 + r8 * 16);
        if (part == 0) dr[row] = __half2float(__ushort_as_half(*(const unsigned short *)(slab + 1664 + r8 * 2)));
        uint4 ql[4], qh[2];
#pragma unroll
        for (int c = 0; c < 4; c++) ql[c] = *(const uint4 *)(slab + (4 * part + c) * 128 + r8 * 16);
#pragma unroll
        for (int c = 0; c < 2; c++) qh[c] = *(const uint4 *)(slab + 1024 + (2 * part + c) * 128 + r8 * 16);
        const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
#pragma unroll
        for (int k = 0; k < 8; k++) {  // the reference's 4-element groups (quant.c:62-74)
            const uint32_t wql[4] = {ql[k >> 2].x, ql[k >> 2].y, ql[k >> 2].z, ql[k >> 2].w};
            const uint32_t wql2[4] = {ql[2 + (k >> 2)].x, ql[2 + (k >> 2)].y, ql[2 + (k >> 2)].z, ql[2 + (k >> 2)].w};
            const uint32_t wqh[4] = {qh[k >> 2].x, qh[k >> 2].y, qh[k >> 2].z, qh[k >> 2].w};
            const uint32_t QL0 = wql[k & 3], QL1 = wql2[k & 3], QH = wqh[k & 3];
            const uint32_t v[4] = {(QL0 & 0x0F0F0F0F) | ((QH << 4) & 0x30303030),
                                   (QL1 & 0x0F0F0F0F) | ((QH << 2) & 0x30303030),
                                   ((QL0 >> 4) & 0x0F0F0F0F) | (QH & 0x30303030),
                                   ((QL1 >> 4) & 0x0F0F0F0F) | ((QH >> 2) & 0x30303030)};
#pragma unroll
            for (int g = 0; g < 4; g++) {  // elements 128p + 32g + 4k + 0..3
                const int e0 = 128 * part + 32 * g + 4 * k;
                const int sc = (int)(int8_t)(scw[e0 >> 6] >> (8 * ((e0 >> 4) & 3)));
                uint32_t hw = 0, lw = 0;
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int prod = sc * ((int)((v[g] >> (8 * i)) & 0xFF) - 32);
                    hw |= (uint32_t)(prod >> 6 & 0xFF) << (8 * i);
                    lw |= (uint32_t)(prod & 63) << (8 * i);
                }
                const int off = plane_off(GM, row, e0);
                *(uint32_t *)(sa + off) = hw;
                *(uint32_t *)(sa + PLANE + off) = lw;
            }
        }
    }
}

struct GemmArgs {
    const uint8_t *slabs;
    int nb;                      // superblocks per row
    int64_t g_begin, g_end;      // weight row groups of the launch
    const int8_t *xqs;           // Q8_K activations of token 0
    const float *xd;
    int qrow, nbx, n_tok;
    float *out;
    int64_t ldo, row0, row1, out_row0;
    const float *residual;
    // Grouped experts (MoE prefill): grid.y walks the work list grp_tiles[0 .. grp_off[ne+1]) of
    // (e << 16 | token tile); expert e's slots are grp_slot[grp_off[e] .. grp_off[e+1]); slot s
    // reads activation row s / xdiv and writes out + s * ldo; expert e's matrix starts at group
    // e * gpe.
    const int32_t *grp_off, *grp_slot, *grp_tiles;
    int n_expert;
    int xdiv;
    int64_t gpe;
    // Split along K (grid.z > 1): CTA z takes superblocks [z * sb_per, (z + 1) * sb_per) and
    // stores term (b, token, row) at terms[(b * n_tok + token) * t_rows + row - g_begin * 8].
    float *terms;
    int64_t t_rows;
    int sb_per;
};

template <int TYPE, bool SPLIT = false>
__global__ void __launch_bounds__(G_THREADS, 1) qgemm_kernel(GemmArgs a) {
    constexpr int NP = GemmPlanes<TYPE>::n;
    constexpr int SB = slab_bytes(TYPE);
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t *sa = smem, *sb = smem + NP * PLANE;  // sb: two B tiles
    float *yd = (float *)(sb + 2 * BTILE), *dr = yd + 2 * GN, *dmr = dr + GM;
    uint8_t *raw = (uint8_t *)(dmr + GM);
    uint64_t *mbar = (uint64_t *)(raw + g_raw_bytes(TYPE));
    uint32_t *tmem_slot = (uint32_t *)(mbar + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t gt0 = a.g_begin + (int64_t)blockIdx.x * (GM / GROUP_ROWS);  // first group of the tile
    int tok0 = blockIdx.y * GN;
    int nv = min(GN, a.n_tok - tok0);
    const uint8_t *slabs = a.slabs;
    const int32_t *gslot = nullptr;  // grouped: the tile's slots
    pdl_wait();
    if (a.grp_off) {
        if ((int)blockIdx.y >= a.grp_off[a.n_expert + 1]) return;  // past the work list: leaves before any barrier
        const int item = a.grp_tiles[blockIdx.y], e = item >> 16;
        tok0 = (item & 0xFFFF) * GN;
        const int g0 = a.grp_off[e];
        nv = min(GN, a.grp_off[e + 1] - g0 - tok0);
        gslot = a.grp_slot + g0 + tok0;
        slabs += (size_t)e * a.gpe * a.nb * slab_bytes(TYPE);
    }
    // activation row and output row of the tile's token t
    auto xrow = [&](int t) -> int64_t { return gslot ? gslot[t] / a.xdiv : tok0 + t; };
    auto orow_of = [&](int t) -> int64_t { return gslot ? gslot[t] : tok0 + t; };

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
    }
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_u32(mbar)));
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    // Padded tokens keep zero activations for the whole kernel.
    for (int i = tid; i < 2 * BTILE / 16; i += G_THREADS)  // chunk-plane layout: i = buffer/plane * GN + t
        if (i % GN >= nv) ((uint4 *)sb)[i] = make_uint4(0, 0, 0, 0);
    for (int i = tid; i < 2 * GN; i += G_THREADS)
        if (i % GN >= nv) yd[i] = 0.0f;
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint32_t mbar_a = smem_u32(mbar);
    const int row = tid & (GM - 1), part = tid >> 7;  // expansion: two threads per weight row
    const int64_t grow = gt0 * GROUP_ROWS + row;        // this thread's weight row
    const bool row_ok = grow < a.g_end * GROUP_ROWS;
    const int erow = (warp & 3) * 32 + lane, ehalf = warp >> 2;  // epilogue: TMEM lane = row, 64 tokens
    float acc[64];
#pragma unroll
    for (int i = 0; i < 64; i++) acc[i] = 0.0f;
    bool ok = true;

    // Superblock b's raw slabs, B tile and token scales, requested with cp.async (B and yd into
    // buffer b & 1) so that they travel while the previous superblock is multiplied.
    const int ng_tile = (int)(a.g_end - gt0 < GM / GROUP_ROWS ? a.g_end - gt0 : GM / GROUP_ROWS);
    // first: the first thread of the copying threads, stride their number (the first superblock's
    // copies by every thread; later ones by warps 1-7 while warp 0 issues the MMAs)
    auto issue = [&](int b, int first) {
        const int me = tid - first, stride = G_THREADS - first;
        if (me >= 0) {
            uint8_t *sbb = sb + (b & 1) * BTILE;
            float *ydb = yd + (b & 1) * GN;
            for (int i = me; i < nv * 16; i += stride) {
                const int t = i >> 4, c = i & 15;
                cp_async16(sbb + c * (GN * 16) + t * 16, a.xqs + (size_t)xrow(t) * a.qrow + b * XQ_SPAN + c * 16);
            }
            for (int t = me; t < nv; t += stride) cp_async4(ydb + t, a.xd + (size_t)xrow(t) * a.nbx + b);
            constexpr int C16 = SB / 16;
            for (int i = me; i < ng_tile * C16; i += stride) {
                const int g = i / C16, c = i - g * C16;
                cp_async16(raw + g * SB + c * 16, slabs + ((size_t)(gt0 + g) * a.nb + b) * SB + c * 16);
            }
        }
        cp_async_commit();
    };
    const int b0 = SPLIT ? (int)blockIdx.z * a.sb_per : 0;
    const int b1 = SPLIT ? min(a.nb, b0 + a.sb_per) : a.nb;
    issue(b0, 0);
    // matrix descriptors of the A planes and of the two B tiles: each MMA adds its constant offset
    // (address / 16 stays far below the field's 14 bits: shared memory is < 256 KB)
    const uint64_t a_desc = kmajor_desc(smem_u32(sa), GM * 16, 128);
    const uint64_t b_desc[2] = {kmajor_desc(smem_u32(sb), GN * 16, 128),
                                kmajor_desc(smem_u32(sb + BTILE), GN * 16, 128)};
    for (int b = b0; b < b1 && ok; b++) {
        cp_async_wait_all();
        __syncthreads();
        if (row_ok) {
            expand_half<TYPE>(raw + (grow / GROUP_ROWS - gt0) * SB, (int)(grow % GROUP_ROWS), row, part, sa, dr, dmr);
        } else {
            for (int k = 128 * part; k < 128 * part + 128; k += 16)
                for (int p = 0; p < NP; p++) *(uint4 *)(sa + p * PLANE + plane_off(GM, row, k)) = make_uint4(0, 0, 0, 0);
            if (part == 0) dr[row] = dmr[row] = 0.0f;
        }
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // B (cp.async) and A for the MMA
        __syncthreads();
        const float *ydb = yd + (b & 1) * GN;
        if (tid == 0) {  // the MMAs first, then the next superblock's copies by warps 1-7 meanwhile
            fence_after_sync();
            const uint32_t idesc = idesc_i8(nv);
            const uint64_t bd0 = b_desc[b & 1];
#pragma unroll
            for (int s = 0; s < 8; s++) {  // K step s: bytes 32s..32s+31 = chunk planes 2s, 2s+1
                const uint64_t bd = bd0 + ((2 * s * GN * 16) >> 4);
#pragma unroll
                for (int p = 0; p < NP; p++)
                    mma_i8(tmem + p * GN, a_desc + ((p * PLANE + 2 * s * GM * 16) >> 4), bd, idesc, s > 0);
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(mbar_a)
                         : "memory");
        }
        if (b + 1 < b1) issue(b + 1, 32);  // the raw buffer is free, B buffer (b+1)&1 was read by MMA b-1
        if (!mbar_wait(mbar_a, (b - b0) & 1)) {
            atomicOr(&g_qgemm_status, 1u);
            ok = false;
        }
        fence_after_sync();
        if (ok) {
            const float d = dr[erow], dm = dmr[erow];
            // split: this row's terms (rows past the matrix's groups store nothing)
            const int64_t trow = (gt0 - a.g_begin) * GROUP_ROWS + erow;
            float *tb = SPLIT && trow < a.t_rows ? a.terms + ((size_t)b * a.n_tok + tok0) * a.t_rows + trow : nullptr;
#pragma unroll
            for (int cc = 0; cc < 2; cc++) {
                const uint32_t col = ehalf * 64 + cc * 32;
                if ((int)col >= nv) continue;  // no valid token in these columns (warp-uniform)
                const uint32_t lanes = (uint32_t)((warp & 3) * 32) << 16;
                int32_t h[32], l[32], m[32];
                tmem_ld32(tmem + lanes + col, h);
                tmem_ld32(tmem + lanes + GN + col, l);
                if constexpr (NP == 3) tmem_ld32(tmem + lanes + 2 * GN + col, m);
                asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    const float y = ydb[col + i];
                    float term;
                    if constexpr (TYPE == T_Q4_K) {
                        const int isum = 32 * h[i] + l[i];
                        const float dall = __fmul_rn(y, d), dmn = __fmul_rn(y, dm);
                        term = __fsub_rn(__fmul_rn(dall, __int2float_rn(isum)), __fmul_rn(dmn, __int2float_rn(m[i])));
                    } else {
                        const int isum = 64 * h[i] + l[i];
                        term = __fmul_rn(__fmul_rn(y, d), __int2float_rn(isum));
                    }
                    if constexpr (SPLIT) {
                        if (tb && (int)(col + i) < nv) tb[(size_t)(col + i) * a.t_rows] = term;
                    } else {
                        acc[cc * 32 + i] = __fadd_rn(acc[cc * 32 + i], term);
                    }
                }
            }
        }
        fence_before_sync();
        __syncthreads();
    }

    cp_async_wait_all();  // nothing in flight when the CTA leaves (only after a timed-out wait)
    // outputs (rows of this tile within [row0, row1), valid tokens)
    const int64_t orow = gt0 * GROUP_ROWS + erow;
    if (ok && !SPLIT && orow >= a.row0 && orow < a.row1) {
#pragma unroll
        for (int i = 0; i < 64; i++) {
            const int t = ehalf * 64 + i;
            if (t < nv) {
                const size_t o = (size_t)orow_of(t) * a.ldo + (orow - a.out_row0);
                a.out[o] = a.residual ? __fadd_rn(a.residual[o], acc[i]) : acc[i];
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        fence_after_sync();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(TMEM_COLS));
    }
}

// out[t][r] (+ residual) = the terms of (r, t) added in superblock order from zero.
__global__ void qgemm_reduce_kernel(const float *terms, int nb, int n_tok, int64_t t_rows, int64_t row_base,
                                    float *out, int64_t ldo, int64_t row0, int64_t row1, int64_t out_row0,
                                    const float *residual) {
    pdl_wait();
    const int64_t r = row0 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int t = blockIdx.y;
    if (r >= row1) return;
    const float *tp = terms + (size_t)t * t_rows + (r - row_base);
    const size_t bstride = (size_t)n_tok * t_rows;
    const float acc = ordered_sum<8>(0.0f, nb, [&](int b) { return __ldcg(tp + (size_t)b * bstride); });
    const size_t o = (size_t)t * ldo + (r - out_row0);
    out[o] = residual ? __fadd_rn(residual[o], acc) : acc;
}

// Stream-ordered pool of the split products' term buffers, one per device, keeping its memory
// between calls (release threshold: unlimited); nullptr when pools are unavailable.
cudaMemPool_t term_pool() {
    static cudaMemPool_t pools[64] = {};
    static std::atomic<int> state[64];  // 0 unset, 1 ready, 2 unavailable
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    int st = state[dev].load();
    if (st == 1) return pools[dev];
    if (st == 2) return nullptr;
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    if (state[dev].load() == 0) {
        cudaMemPoolProps props = {};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = dev;
        cudaMemPool_t p = nullptr;
        uint64_t keep = ~0ull;
        if (cudaMemPoolCreate(&p, &props) == cudaSuccess &&
            cudaMemPoolSetAttribute(p, cudaMemPoolAttrReleaseThreshold, &keep) == cudaSuccess) {
            pools[dev] = p;
            state[dev].store(1);
        } else {
            cudaGetLastError();
            state[dev].store(2);
        }
    }
    return state[dev].load() == 1 ? pools[dev] : nullptr;
}

int device_sms() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    return n;
}

// ------------------------------------------------------------------- 32-element block formats
constexpr int KB = 4;                  // blocks per step (one TMEM accumulator each)
constexpr int APLANE32 = GM * 32;      // A bytes of one block
constexpr int BTILE32 = GN * 32 * KB;  // B bytes of one step

__host__ __device__ constexpr int g32_raw_bytes(int type) { return (GM / GROUP_ROWS) * KB * slab_bytes(type); }
__host__ __device__ constexpr int g32_smem_bytes(int type) {
    return KB * APLANE32 + 2 * BTILE32 + 2 * KB * GN * 4 + KB * GM * 4 + g32_raw_bytes(type) + 16;
}

// One (row, block) of the A tile: the 32 values (bias removed) as two 16-byte K chunks of the
// block's plane, and the row's block scale. slab: the (row group, block) slab; r8: row in group.
template <int TYPE>
__device__ __forceinline__ void expand_block32(const uint8_t *slab, int r8, int row, uint8_t *plane, float *dw) {
    uint4 lo, hi;
    if constexpr (TYPE == T_Q8_0) {
        lo = *(const uint4 *)(slab + r8 * 16);
        hi = *(const uint4 *)(slab + 128 + r8 * 16);
        *dw = __half2float(__ushort_as_half(*(const unsigned short *)(slab + 256 + r8 * 2)));
    } else {
        // element e < 16: low nibble of byte e; e >= 16: high nibble of byte e - 16 (Q5_0: bit e
        // of qh above it)
        const uint4 q = *(const uint4 *)(slab + r8 * 16);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
        uint32_t qh = 0;
        if constexpr (TYPE == T_Q5_0) qh = *(const uint32_t *)(slab + 128 + r8 * 4);
        constexpr uint32_t bias = TYPE == T_Q4_0 ? 0x08080808u : 0x10101010u;
        uint32_t l[4], h[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            l[k] = w[k] & 0x0F0F0F0Fu;
            h[k] = (w[k] >> 4) & 0x0F0F0F0Fu;
            if constexpr (TYPE == T_Q5_0) {
                l[k] |= ((((qh >> (4 * k)) & 15u) * 0x00204081u) & 0x01010101u) << 4;
                h[k] |= ((((qh >> (16 + 4 * k)) & 15u) * 0x00204081u) & 0x01010101u) << 4;
            }
            l[k] = __vsub4(l[k], bias);  // bytewise, no borrow between bytes
            h[k] = __vsub4(h[k], bias);
        }
        lo = make_uint4(l[0], l[1], l[2], l[3]);
        hi = make_uint4(h[0], h[1], h[2], h[3]);
        *dw = __half2float(__ushort_as_half(*(const unsigned short *)(slab + (TYPE == T_Q4_0 ? 128 : 160) + r8 * 2)));
    }
    *(uint4 *)(plane + plane_off(GM, row, 0)) = lo;
    *(uint4 *)(plane + plane_off(GM, row, 16)) = hi;
}

template <int TYPE>
__global__ void __launch_bounds__(G_THREADS, 1) qgemm32_kernel(GemmArgs a) {
    constexpr int SB = slab_bytes(TYPE);
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t *sa = smem, *sb = smem + KB * APLANE32;  // sa: KB block planes, sb: two B tiles
    float *yd = (float *)(sb + 2 * BTILE32);         // [2][KB][GN] token block scales
    float *dwr = yd + 2 * KB * GN;                   // [KB][GM] row block scales
    uint8_t *raw = (uint8_t *)(dwr + KB * GM);       // [groups][KB] slabs of the next step
    uint64_t *mbar = (uint64_t *)(raw + g32_raw_bytes(TYPE));
    uint32_t *tmem_slot = (uint32_t *)(mbar + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t gt0 = a.g_begin + (int64_t)blockIdx.x * (GM / GROUP_ROWS);
    int tok0 = blockIdx.y * GN;
    int nv = min(GN, a.n_tok - tok0);
    const uint8_t *slabs = a.slabs;
    const int32_t *gslot = nullptr;
    pdl_wait();
    if (a.grp_off) {
        if ((int)blockIdx.y >= a.grp_off[a.n_expert + 1]) return;
        const int item = a.grp_tiles[blockIdx.y], e = item >> 16;
        tok0 = (item & 0xFFFF) * GN;
        const int g0 = a.grp_off[e];
        nv = min(GN, a.grp_off[e + 1] - g0 - tok0);
        gslot = a.grp_slot + g0 + tok0;
        slabs += (size_t)e * a.gpe * a.nb * SB;
    }
    auto xrow = [&](int t) -> int64_t { return gslot ? gslot[t] / a.xdiv : tok0 + t; };
    auto orow_of = [&](int t) -> int64_t { return gslot ? gslot[t] : tok0 + t; };

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
    }
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_u32(mbar)));
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    for (int i = tid; i < 2 * BTILE32 / 16; i += G_THREADS)  // padded tokens: zero activations
        if (i % GN >= nv) ((uint4 *)sb)[i] = make_uint4(0, 0, 0, 0);
    for (int i = tid; i < 2 * KB * GN; i += G_THREADS)
        if (i % GN >= nv) yd[i] = 0.0f;
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint32_t mbar_a = smem_u32(mbar);
    const int row = tid & (GM - 1), part = tid >> 7;  // expansion: blocks 2*part, 2*part+1 of a row
    const int64_t grow = gt0 * GROUP_ROWS + row;
    const bool row_ok = grow < a.g_end * GROUP_ROWS;
    const int erow = (warp & 3) * 32 + lane, ehalf = warp >> 2;  // epilogue: TMEM lane = row, 64 tokens
    float acc[64];
#pragma unroll
    for (int i = 0; i < 64; i++) acc[i] = 0.0f;
    bool ok = true;

    const int ng_tile = (int)(a.g_end - gt0 < GM / GROUP_ROWS ? a.g_end - gt0 : GM / GROUP_ROWS);
    const int steps = (a.nb + KB - 1) / KB;
    // Step s: blocks KB*s .. KB*s + nblk - 1 (elements 128s.., inside one 256-element XQ span).
    // first: as in qgemm_kernel (warp 0 issues the MMAs while warps 1-7 copy the next step)
    auto issue = [&](int st, int first) {
        const int me = tid - first, stride = G_THREADS - first;
        if (me >= 0) {
            const int b0 = st * KB, nblk = min(KB, a.nb - b0), chunks = 2 * nblk;
            uint8_t *sbb = sb + (st & 1) * BTILE32;
            float *ydb = yd + (st & 1) * KB * GN;
            for (int i = me; i < nv * chunks; i += stride) {
                const int t = i / chunks, c = i - t * chunks;
                cp_async16(sbb + c * (GN * 16) + t * 16, a.xqs + (size_t)xrow(t) * a.qrow + xq_pos(32 * b0) + c * 16);
            }
            for (int i = me; i < nv * nblk; i += stride) {
                const int t = i / nblk, j = i - t * nblk;
                cp_async4(ydb + j * GN + t, a.xd + (size_t)xrow(t) * a.nbx + b0 + j);
            }
            constexpr int C16 = SB / 16;
            for (int i = me; i < ng_tile * nblk * C16; i += stride) {
                const int gj = i / C16, c = i - gj * C16, g = gj / nblk, j = gj - g * nblk;
                cp_async16(raw + (g * KB + j) * SB + c * 16,
                           slabs + ((size_t)(gt0 + g) * a.nb + b0 + j) * SB + c * 16);
            }
        }
        cp_async_commit();
    };
    issue(0, 0);
    for (int st = 0; st < steps && ok; st++) {
        const int nblk = min(KB, a.nb - st * KB);
        cp_async_wait_all();
        __syncthreads();
#pragma unroll
        for (int jj = 0; jj < 2; jj++) {
            const int j = 2 * part + jj;
            if (j < nblk) {
                if (row_ok) {
                    expand_block32<TYPE>(raw + ((grow / GROUP_ROWS - gt0) * KB + j) * SB, (int)(grow % GROUP_ROWS), row,
                                         sa + j * APLANE32, dwr + j * GM + row);
                } else {
                    *(uint4 *)(sa + j * APLANE32 + plane_off(GM, row, 0)) = make_uint4(0, 0, 0, 0);
                    *(uint4 *)(sa + j * APLANE32 + plane_off(GM, row, 16)) = make_uint4(0, 0, 0, 0);
                    dwr[j * GM + row] = 0.0f;
                }
            }
        }
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        __syncthreads();
        const uint8_t *sbb = sb + (st & 1) * BTILE32;
        const float *ydb = yd + (st & 1) * KB * GN;
        if (tid == 0) {
            fence_after_sync();
            const uint32_t idesc = idesc_i8(nv);
            for (int j = 0; j < nblk; j++)
                mma_i8(tmem + j * GN, kmajor_desc(smem_u32(sa + j * APLANE32), GM * 16, 128),
                       kmajor_desc(smem_u32(sbb + 2 * j * GN * 16), GN * 16, 128), idesc, 0);
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(mbar_a)
                         : "memory");
        }
        if (st + 1 < steps) issue(st + 1, 32);  // raw is free; B buffer (st+1)&1 was read by MMA st-1
        if (!mbar_wait(mbar_a, st & 1)) {
            atomicOr(&g_qgemm_status, 1u);
            ok = false;
        }
        fence_after_sync();
        if (ok) {
            const uint32_t lanes = (uint32_t)((warp & 3) * 32) << 16;
            for (int j = 0; j < nblk; j++) {  // block order
                const float dw = dwr[j * GM + erow];
#pragma unroll
                for (int cc = 0; cc < 2; cc++) {
                    const uint32_t col = ehalf * 64 + cc * 32;
                    if ((int)col >= nv) continue;  // no valid token in these columns (warp-uniform)
                    int32_t v[32];
                    tmem_ld32(tmem + lanes + j * GN + col, v);
                    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
                    for (int i = 0; i < 32; i++)  // (float)s * (dw * dx), quant.c:160
                        acc[cc * 32 + i] = __fadd_rn(acc[cc * 32 + i],
                                                     __fmul_rn(__int2float_rn(v[i]), __fmul_rn(dw, ydb[j * GN + col + i])));
                }
            }
        }
        fence_before_sync();
        __syncthreads();
    }

    cp_async_wait_all();
    const int64_t orow = gt0 * GROUP_ROWS + erow;
    if (ok && orow >= a.row0 && orow < a.row1) {
#pragma unroll
        for (int i = 0; i < 64; i++) {
            const int t = ehalf * 64 + i;
            if (t < nv) {
                const size_t o = (size_t)orow_of(t) * a.ldo + (orow - a.out_row0);
                a.out[o] = a.residual ? __fadd_rn(a.residual[o], acc[i]) : acc[i];
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        fence_after_sync();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(TMEM_COLS));
    }
}

bool is_block32(int type) { return type == T_Q8_0 || type == T_Q4_0 || type == T_Q5_0; }

// The kernel of the weight type, with its shared memory (a.terms set: the split K-quant kernel).
void launch_gemm(int type, dim3 grid, const GemmArgs &a, cudaStream_t s) {
    if (a.terms) {
        if (type == T_Q4_K) {
            static std::atomic<uint64_t> configured{0};
            smem_limit_once(qgemm_kernel<T_Q4_K, true>, g_smem_bytes(3, T_Q4_K), configured);
            launch(qgemm_kernel<T_Q4_K, true>, grid, G_THREADS, g_smem_bytes(3, T_Q4_K), s, a);
        } else {
            static std::atomic<uint64_t> configured{0};
            smem_limit_once(qgemm_kernel<T_Q6_K, true>, g_smem_bytes(2, T_Q6_K), configured);
            launch(qgemm_kernel<T_Q6_K, true>, grid, G_THREADS, g_smem_bytes(2, T_Q6_K), s, a);
        }
        SDY_LAUNCHED();
        return;
    }
    switch (type) {
#define SDY_GEMM_CASE(T, KERNEL, SMEM)                          \
    case T: {                                                   \
        static std::atomic<uint64_t> configured{0};            \
        smem_limit_once(KERNEL<T>, SMEM, configured);           \
        launch(KERNEL<T>, grid, G_THREADS, SMEM, s, a);         \
        break;                                                  \
    }
        SDY_GEMM_CASE(T_Q4_K, qgemm_kernel, g_smem_bytes(3, T_Q4_K))
        SDY_GEMM_CASE(T_Q6_K, qgemm_kernel, g_smem_bytes(2, T_Q6_K))
        SDY_GEMM_CASE(T_Q8_0, qgemm32_kernel, g32_smem_bytes(T_Q8_0))
        SDY_GEMM_CASE(T_Q4_0, qgemm32_kernel, g32_smem_bytes(T_Q4_0))
        SDY_GEMM_CASE(T_Q5_0, qgemm32_kernel, g32_smem_bytes(T_Q5_0))
#undef SDY_GEMM_CASE
    default: set_error("qgemm: weight type %d has no tensor-core kernel", type); return;
    }
    SDY_LAUNCHED();
}

}  // namespace

bool qgemm_supported(int type, int n_in) {
    return ((type == T_Q4_K || type == T_Q6_K) && n_in % 256 == 0) || (is_block32(type) && n_in % 32 == 0);
}

// The activation layout the weight type multiplies with (Q8_K for the K-quants, Q8_0 otherwise).
static int gemm_vtype(int type) { return is_block32(type) ? T_Q8_0 : T_Q8_K; }

void qgemm(const QMat &w, const XQ &xq, float *out, int64_t ldo, int64_t row0, int64_t row1, int64_t out_row0,
           cudaStream_t s, const float *residual, bool split_ok) {
    if (row1 <= row0 || xq.n_tok <= 0) return;
    if (!qgemm_supported(w.type, w.n_in) || xq.vtype != gemm_vtype(w.type) || xq.n_in != w.n_in) {
        set_error("qgemm: unsupported weight type %d / activation layout", w.type);
        return;
    }
    GemmArgs a{};
    a.slabs = w.slabs;
    a.nb = w.nb;
    a.g_begin = row0 / GROUP_ROWS;
    a.g_end = (row1 + GROUP_ROWS - 1) / GROUP_ROWS;
    a.xqs = xq.qs;
    a.xd = xq.d;
    a.qrow = xq.qrow;
    a.nbx = xq.nbx;
    a.n_tok = xq.n_tok;
    a.out = out;
    a.ldo = ldo;
    a.row0 = row0;
    a.row1 = row1;
    a.out_row0 = out_row0;
    a.residual = residual;
    const int64_t tiles_m = (a.g_end - a.g_begin + GM / GROUP_ROWS - 1) / (GM / GROUP_ROWS);
    const int64_t tiles_n = (xq.n_tok + GN - 1) / GN;
    // Split along K where a simple cost model says it pays: a tile's superblock takes about
    // SB_US (one CTA per SM), the term buffer is written and read once more at about 3 TB/s
    // (both measured on B200), and the reduction costs a launch. At least 2 superblocks per CTA,
    // a term buffer of at most 1 GiB, never inside a stream capture.
    const int sms = device_sms();
    int splits = 1;
    const int64_t tiles = tiles_m * tiles_n;
    static const bool split_off = [] {  // SARDYNE_GEMM_SPLIT=off: one CTA per tile always
        const char *v = getenv("SARDYNE_GEMM_SPLIT");
        return v && !strcmp(v, "off");
    }();
    if (split_ok && !split_off && !is_block32(w.type) && tiles < sms && w.nb >= 4) {
        constexpr double SB_US = 3.0, TERM_GBS = 3000.0, REDUCE_US = 3.0;
        const int64_t t_rows = (a.g_end - a.g_begin) * GROUP_ROWS;
        const double term_us = 2.0 * (double)w.nb * xq.n_tok * t_rows * 4 / (TERM_GBS * 1e3);
        double best = (double)((tiles + sms - 1) / sms) * w.nb * SB_US;
        for (int sp = 2; sp <= w.nb / 2; sp++) {
            const int per = (w.nb + sp - 1) / sp;
            const double t = (double)((tiles * sp + sms - 1) / sms) * per * SB_US + term_us + REDUCE_US;
            if (t < best) best = t, splits = sp;
        }
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        if ((size_t)w.nb * xq.n_tok * t_rows * 4 > ((size_t)1 << 30) || cudaStreamIsCapturing(s, &cap) != cudaSuccess ||
            cap != cudaStreamCaptureStatusNone)
            splits = 1;
    }
    cudaMemPool_t pool = splits > 1 ? term_pool() : nullptr;
    float *terms = nullptr;
    if (pool) {
        a.t_rows = (a.g_end - a.g_begin) * GROUP_ROWS;
        const size_t bytes = (size_t)w.nb * xq.n_tok * a.t_rows * 4;
        if (cudaMallocFromPoolAsync((void **)&terms, bytes, pool, s) != cudaSuccess) {
            cudaGetLastError();  // no scratch: one CTA per tile after all
            terms = nullptr;
        }
    }
    if (!terms) {
        launch_gemm(w.type, dim3((unsigned)tiles_m, (unsigned)tiles_n), a, s);
        return;
    }
    a.terms = terms;
    a.sb_per = (w.nb + splits - 1) / splits;
    const int nz = (w.nb + a.sb_per - 1) / a.sb_per;
    launch_gemm(w.type, dim3((unsigned)tiles_m, (unsigned)tiles_n, (unsigned)nz), a, s);
    launch(qgemm_reduce_kernel, dim3((unsigned)((row1 - row0 + 255) / 256), (unsigned)xq.n_tok), 256, 0, s,
           (const float *)terms, w.nb, xq.n_tok, a.t_rows, a.g_begin * GROUP_ROWS, out, ldo, row0, row1, out_row0,
           residual);
    SDY_LAUNCHED();
    SDY_CUDA(cudaFreeAsync(terms, s));
}

void qgemm_grouped(const QMat &experts, int64_t gpe, int n_expert, const XQ &xq, int xdiv, const int32_t *grp_off,
                   const int32_t *grp_slot, const int32_t *grp_tiles, int max_slots, int64_t rows_per_expert,
                   float *out, int64_t ldo_slot, cudaStream_t s) {
    if (max_slots <= 0 || n_expert <= 0) return;
    if (!qgemm_supported(experts.type, experts.n_in) || xq.vtype != gemm_vtype(experts.type) ||
        xq.n_in != experts.n_in) {
        set_error("qgemm_grouped: unsupported weight type %d / activation layout", experts.type);
        return;
    }
    GemmArgs a{};
    a.slabs = experts.slabs;
    a.nb = experts.nb;
    a.g_begin = 0;
    a.g_end = (rows_per_expert + GROUP_ROWS - 1) / GROUP_ROWS;
    a.xqs = xq.qs;
    a.xd = xq.d;
    a.qrow = xq.qrow;
    a.nbx = xq.nbx;
    a.n_tok = max_slots;
    a.out = out;
    a.ldo = ldo_slot;
    a.row0 = 0;
    a.row1 = rows_per_expert;
    a.out_row0 = 0;
    a.grp_off = grp_off;
    a.grp_slot = grp_slot;
    a.grp_tiles = grp_tiles;
    a.n_expert = n_expert;
    a.xdiv = xdiv;
    a.gpe = gpe;
    const int64_t tiles_m = (a.g_end + GM / GROUP_ROWS - 1) / (GM / GROUP_ROWS);
    // at most ceil(count_e / GN) tiles per expert: sum <= max_slots / GN + n_expert
    const dim3 grid((unsigned)tiles_m, (unsigned)(max_slots / GN + n_expert));
    launch_gemm(experts.type, grid, a, s);
}

unsigned qgemm_status() {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_qgemm_status, sizeof v) != cudaSuccess) return ~0u;
    return v;
}

void qgemm_clear_status() {
    const unsigned z = 0;
    SDY_CUDA(cudaMemcpyToSymbol(g_qgemm_status, &z, sizeof z));
}

}  // namespace sdy
