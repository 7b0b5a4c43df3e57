// The prefill expert GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), reading the raw GGUF blocks.
//
// Per tile: 128 weight rows of one expert (the MMA's A operand, M = 128) x up to 256 of the expert's (token, slot)
// rows in dispatch order (B, N <= 256), K in stages of 64, an fp32 accumulator in TMEM (two of 256 columns: the
// epilogue of tile i overlaps the MMAs of tile i + 1). D = A . B^T, so the output rows are weight rows and its
// columns tokens; the epilogue transposes on the way out.
//   gu    A = 64 gate rows and the 64 up rows of the same features, arranged so that every epilogue warp holds 16 gate
//         and the matching 16 up rows (TMEM lanes 32q + l: l < 16 gate feature 16q + l, l >= 16 up feature 16q + l - 16);
//         out h[(token), f] = silu(g) u in bf16 (ref.swiglu, tests/moe/ref.py:21-24).
//   down  A = 128 down rows; out y[(token), n] in bf16.
// Warp roles (480 threads, one CTA per SM or one two-CTA cluster per SM pair, persistent over a static round-robin of
// tiles):
//   warp 0      TMA producer: raw weight bytes (2D tensor map over the GGUF rows, 16-bit elements, 256 K-values
//               per stage: 144 B a row for Q4_0 / Q4_K / IQ4_NL, 160 B for Q4_1, 176 B for Q5_K, 272 B for Q8_0) and
//               the token rows (bf16, 128-byte swizzle); it also allocates and frees the 512 TMEM columns.
//   warp 1      MMA issuer: tcgen05.mma kind::f16 (bf16 x bf16 -> fp32), one thread; tcgen05.commit frees stages.
//   warps 2-9   dequant, every warp on every step in step order: thread (h, i) decodes values 32 h .. 32 h + 31 of
//               A row i of each 64-value step (h = 0 for warps 2-5, 1 for warps 6-9) from only that block's raw bytes;
//               the reference's exact fp32 values (magic-number byte conversion, f32x2 arithmetic), rounded once to
//               bf16, written into the A stage in the UMMA K-major 128-byte-swizzle layout; fence.proxy.async, then
//               every lane arrives on the stage's full barrier. A stage's writers wait on every phase of its empty
//               barrier in order (a parity wait that skipped phases would have to infer them from other barriers,
//               whose arrivals from the tensor core are not ordered for an observer).
//   warps 10-13 epilogue: tcgen05.ld of 32 columns at a time, SwiGLU (gu) or the plain rows (down), bf16 stores.
//   warp 14     (Q6_K, Q3_K, IQ4_XS) the copy warp: rows of 210 / 110 / 136 B a super-block are not 16-byte pitched,
//               so no tensor map describes them; 16-byte cp.async copies of each row's 16-byte-aligned window instead.
// Every mbarrier wait is bounded (kWaitCycles): on expiry the CTA records ARTLITE_ETIMEOUT in the status word, stops
// issuing, lets copies and MMAs already issued land, frees its TMEM and exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "kernels.cuh"
#include "quant.cuh"
#include "tc_gemm.cuh"


namespace artlite {
namespace tc {

constexpr int BM = 128, BNMAX = 256, BK = 64, KC = 256, SMAX = 5, RMAX = 3;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BNMAX * BK * 2;
constexpr int kThreads = 480;  // 15 warps: producer, MMA, 8 dequant, 4 epilogue, the Q6_K copy warp
constexpr long long kWaitCycles = 4000000000LL;  // ~2 s at the B200's clocks

__host__ __device__ constexpr int chunk_bytes(int qt) {  // raw bytes of 256 values of a row
  return qt == ARTLITE_Q8_0 ? 272 : (qt == ARTLITE_Q4_0 || qt == ARTLITE_Q4_K || qt == ARTLITE_IQ4_NL) ? 144
       : qt == ARTLITE_Q5_K ? 176 : qt == ARTLITE_Q6_K ? 210 : qt == ARTLITE_Q3_K ? 110 : qt == ARTLITE_IQ4_XS ? 136
       : qt == ARTLITE_Q4_1 ? 160 : 0;
}
// a raw stage row in shared memory: the chunk's bytes (TMA formats), or for Q6_K (whose rows need not be 16-byte
// pitched, so no tensor map can describe them) the 16-byte-aligned 224-byte window around the 210-byte super-block,
// copied by the copy warp, in rows 240 bytes apart (16-byte loads of 8 consecutive rows fall in distinct banks)
__host__ __device__ constexpr int raw_pitch(int qt) {
  return qt == ARTLITE_Q6_K ? 240 : qt == ARTLITE_Q3_K ? 144 : qt == ARTLITE_IQ4_XS ? 176 : chunk_bytes(qt);
}
// the formats whose rows the copy warp brings (Q6_K, 210 B, Q3_K, 110 B, IQ4_XS, 136 B a super-block: rows need not be
// 16-byte pitched), and the 16-byte copies of a row's window (the block plus the up to 14 bytes before it from the
// 16-byte boundary at or below its start: Q6_K 224 bytes, Q3_K 128, IQ4_XS 160)
__host__ __device__ constexpr bool windowed(int qt) {
  return qt == ARTLITE_Q6_K || qt == ARTLITE_Q3_K || qt == ARTLITE_IQ4_XS;
}
__host__ __device__ constexpr int window_chunks(int qt) {
  return qt == ARTLITE_Q6_K ? 14 : qt == ARTLITE_Q3_K ? 8 : qt == ARTLITE_IQ4_XS ? 10 : 0;
}

// raw weight stages: three of 18 KB for the 144-byte formats, two of 34 KB for Q8_0 (shared memory)
__host__ __device__ constexpr int raw_stages(int qt) { return qt == ARTLITE_Q8_0 || qt == ARTLITE_Q6_K ? 2 : 3; }

struct Params {
  CUtensorMap map_w0, map_w1, map_x;
  const uint8_t* gw0;  // the raw rows in global memory (gate / down; up), for the Q6_K copy warp
  const uint8_t* gw1;
  int64_t rb;          // their row bytes
  int cb;              // raw bytes of 256 values (a super-block)
  const int64_t* offsets;
  const int32_t* wexp;  // (may be null) the weight expert of each row group
  const int32_t* toff;  // [E + 1] tiles per expert (ceil(n_e / 256) * MT), scanned
  uint16_t* out;
  DevStatus* status;
  int E, K, N, MT;
};

struct Smem {
  uint64_t full_a[SMAX], full_b[SMAX], empty[SMAX], raw_full[RMAX], raw_empty[RMAX], tfull[2], tempty[2];
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// a bounded wait: false once the CTA aborted (this wait ran out, or another role's did)
__device__ __forceinline__ bool wait(int* abort, uint64_t* bar, uint32_t parity, DevStatus* st, int where) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*(volatile int*)abort) return false;
    if (clock64() - t0 > kWaitCycles) {
      *(volatile int*)abort = 1;
      report(st, ARTLITE_ETIMEOUT, where, (int)blockIdx.x, 0);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart (SBO), version 1
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// instruction descriptor: kind::f16, A = B = bf16, D = f32, both K-major, M x N
__device__ __forceinline__ uint32_t idesc(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(id), "r"(acc));
}
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// a 32-lane x 32-column TMEM load, asynchronous: its registers are valid after tmem_wait32 on the same array (the
// wait names them as operands, so no use of them moves above it)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait32(uint32_t (&v)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15]),
                 "+r"(v[16]), "+r"(v[17]), "+r"(v[18]), "+r"(v[19]), "+r"(v[20]), "+r"(v[21]), "+r"(v[22]),
                 "+r"(v[23]), "+r"(v[24]), "+r"(v[25]), "+r"(v[26]), "+r"(v[27]), "+r"(v[28]), "+r"(v[29]),
                 "+r"(v[30]), "+r"(v[31])
               :
               : "memory");
}

struct Tile {
  int e, m;
  int we;        // the weight expert of row group e
  int64_t row0;  // dispatch row of the tile's first token
  int valid;     // tokens in the tile
  int n_mma;     // MMA N: valid rounded up to 16
};

__device__ __forceinline__ Tile tile_of(const Params& p, int t) {
  int lo = 0, hi = p.E;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (p.toff[mid] <= t) lo = mid; else hi = mid;
  }
  const int local = t - p.toff[lo];
  const int j = local / p.MT;
  Tile T;
  T.e = lo;
  T.we = p.wexp ? p.wexp[lo] : lo;
  T.m = local % p.MT;
  const int64_t o = p.offsets[lo];
  const int n_e = (int)(p.offsets[lo + 1] - o);
  const int ntile = (n_e + BNMAX - 1) / BNMAX;
  const int tile_n = (((n_e + ntile - 1) / ntile) + 15) & ~15;
  const int start = j * tile_n;
  T.row0 = o + start;
  T.valid = min(n_e - start, tile_n);
  T.n_mma = (T.valid + 15) & ~15;
  return T;
}

// the global address of raw row `row` (of the tile's 128) for 256-value chunk kc
template <bool GU>
__device__ __forceinline__ uintptr_t raw_src(const Params& p, const Tile& T, int npeer, uint32_t crank, int row, int kc) {
  const int m = npeer * T.m + (int)crank;
  const uint8_t* base;
  int64_t r;
  if (GU) {  // (gate / up: rows 0-63 gate, 64-127 up, of this CTA's 64 features)
    base = row < 64 ? p.gw0 : p.gw1;
    r = (int64_t)T.we * p.N + 64 * m + (row & 63);
  } else {
    base = p.gw0;
    r = (int64_t)T.we * p.N + BM * m + row;
  }
  return reinterpret_cast<uintptr_t>(base + r * p.rb + (int64_t)kc * p.cb);
}

// ---------------------------------------------------------------- dequant of one 64-value step into bf16 pairs
//
// Exact integer -> fp32 by the "magic number": a byte b placed under the exponent of 2^23 (0x4B000000 | b) is the
// float 2^23 + b, and subtracting 2^23 (+ an offset) leaves b (- the offset) exactly. Byte selection is one PRMT per
// value; the fp32 arithmetic runs on f32x2 pairs (two values an instruction); each value is then the reference's fp32
// result exactly (the same products / differences, rounded to nearest once each, no FMA) before its one rounding to
// bf16.

__device__ __forceinline__ uint32_t byte_at(const uint32_t* w, int b) { return (w[b >> 2] >> ((b & 3) * 8)) & 0xFFu; }
__device__ __forceinline__ float half_at(const uint32_t* w, int b) {
  const uint32_t v = (b & 3) == 0 ? (w[b >> 2] & 0xFFFFu) : (b & 3) == 2 ? (w[b >> 2] >> 16)
                                                                         : (byte_at(w, b) | (byte_at(w, b + 1) << 8));
  return __half2float(__ushort_as_half((unsigned short)v));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
// the 4 bytes of w as the floats 2^23 + byte, in pairs
__device__ __forceinline__ void magic4(uint32_t w, uint64_t& p01, uint64_t& p23) {
  const uint32_t a = __byte_perm(w, 0x4B00u, 0x5440), b = __byte_perm(w, 0x4B00u, 0x5441);
  const uint32_t c = __byte_perm(w, 0x4B00u, 0x5442), d = __byte_perm(w, 0x4B00u, 0x5443);
  asm("mov.b64 %0, {%1, %2};" : "=l"(p01) : "r"(a), "r"(b));
  asm("mov.b64 %0, {%1, %2};" : "=l"(p23) : "r"(c), "r"(d));
}
__device__ __forceinline__ uint64_t dup2(float v) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %1};" : "=l"(r) : "f"(v));
  return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
// bytes i and j of w, each placed in byte kPos (1 or 2) of a word whose byte 3 is kExp and whose other bytes are 0:
// with kExp the top byte of the float 2^E (its exponent's low bit 0), the floats 2^E + byte 2^(E - 23 + 8 kPos)
template <uint32_t kExp, int kPos>
__device__ __forceinline__ uint64_t under2(uint32_t w, int i, int j) {
  // selector nibbles: kPos takes byte i (j) of w, byte 3 takes operand byte 4 (kExp), the rest operand byte 5 (0)
  const uint32_t si = kPos == 1 ? (0x4505u | (uint32_t)i << 4) : (0x4055u | (uint32_t)i << 8);
  const uint32_t sj = kPos == 1 ? (0x4505u | (uint32_t)j << 4) : (0x4055u | (uint32_t)j << 8);
  const uint32_t a = __byte_perm(w, kExp, si), b = __byte_perm(w, kExp, sj);
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf16x2(uint64_t v) {
  float a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
  return pack_bf16(a, b);
}
// the 16 bytes starting at byte o (o even) of w as 4 words
__device__ __forceinline__ void words16(const uint32_t* w, int o, uint32_t (&q)[4]) {
#pragma unroll
  for (int k = 0; k < 4; k++)
    q[k] = (o & 2) ? __funnelshift_r(w[(o >> 2) + k], w[(o >> 2) + k + 1], 16) : w[(o >> 2) + k];
}

// Q4_0 block at byte o of the stage's row bytes: 32 values (q - 8) d as 16 bf16 pairs into o16. A low nibble q in
// byte 2 under the exponent byte 0x43 is the float 128 + q; a high nibble left in place (bits 4-7 of byte 1) under
// 0x45 is 2048 + q. One fused multiply-add a pair, (128 + q) d - 136 d or (2048 + q) d - 2056 d, is (q - 8) d
// exactly: 136 d and 2056 d are exact products (at most 20 significant bits), and so is the single rounding of the
// exact result (q - 8) d (at most 15 bits); then one rounding to bf16, as the reference's fp32 value rounded
__device__ __forceinline__ void dq_q4_0_block(const uint32_t* w, int o, uint32_t* o16) {
  const float df = half_at(w, o);
  const uint64_t d = dup2(df), clo = dup2(-136.0f * df), chi = dup2(-2056.0f * df);
  uint32_t q[4];
  words16(w, o + 2, q);
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const uint32_t lo = q[k] & 0x0F0F0F0Fu, hi = q[k] & 0xF0F0F0F0u;
    o16[2 * k] = bf16x2(fma2(under2<0x43u, 2>(lo, 0, 1), d, clo));  // values 4k, 4k + 1 (low nibbles)
    o16[2 * k + 1] = bf16x2(fma2(under2<0x43u, 2>(lo, 2, 3), d, clo));
    o16[8 + 2 * k] = bf16x2(fma2(under2<0x45u, 1>(hi, 0, 1), d, chi));  // values 16 + 4k, .. (high nibbles)
    o16[8 + 2 * k + 1] = bf16x2(fma2(under2<0x45u, 1>(hi, 2, 3), d, chi));
  }
}

// Q4_1 block at byte o (dequant.cpp:49-56: 20 B per 32, d, m, then Q4_0's nibble layout): 32 values d q + m (a product
// and a sum, each rounded once)
__device__ __forceinline__ void dq_q4_1_block(const uint32_t* w, int o, uint32_t* o16) {
  const uint64_t d = dup2(half_at(w, o)), m = dup2(half_at(w, o + 2)), off = dup2(-8388608.0f);  // -2^23
  uint32_t q[4];
  words16(w, o + 4, q);
#pragma unroll
  for (int k = 0; k < 4; k++) {
    uint64_t a, b, c, e;
    magic4(q[k] & 0x0F0F0F0Fu, a, b);
    magic4((q[k] >> 4) & 0x0F0F0F0Fu, c, e);
    o16[2 * k] = bf16x2(add2(mul2(d, add2(a, off)), m));
    o16[2 * k + 1] = bf16x2(add2(mul2(d, add2(b, off)), m));
    o16[8 + 2 * k] = bf16x2(add2(mul2(d, add2(c, off)), m));
    o16[8 + 2 * k + 1] = bf16x2(add2(mul2(d, add2(e, off)), m));
  }
}

// Q8_0 block at byte o: 32 values d q (q int8: biased by 128 into a byte, then the magic). (Q4_0's fused
// multiply-add form, (32768 + b) d - 32896 d, is exact here too, but measured slower: config 3 0.596 -> 0.64 ms.)
__device__ __forceinline__ void dq_q8_0_block(const uint32_t* w, int o, uint32_t* o16) {
  const uint64_t d = dup2(half_at(w, o)), off = dup2(-8388736.0f);  // -(2^23 + 128)
#pragma unroll
  for (int h = 0; h < 2; h++) {
    uint32_t q[4];
    words16(w, o + 2 + 16 * h, q);
#pragma unroll
    for (int k = 0; k < 4; k++) {
      uint64_t a, b;
      magic4(q[k] ^ 0x80808080u, a, b);
      o16[8 * h + 2 * k] = bf16x2(mul2(d, add2(a, off)));
      o16[8 * h + 2 * k + 1] = bf16x2(mul2(d, add2(b, off)));
    }
  }
}

// Q4_K group g of the stage's super-block: 32 values q (d sc_g) - dmin mn_g
__device__ __forceinline__ void dq_q4_k_group(const uint32_t* w, int g, uint32_t* o16) {
  const float d = half_at(w, 0), dmin = half_at(w, 2);
  int sc, mn;
  if (g < 4) {
    sc = byte_at(w, 4 + g) & 63;
    mn = byte_at(w, 8 + g) & 63;
  } else {
    sc = (byte_at(w, 12 + g - 4) & 15) | (byte_at(w, 4 + g - 4) >> 6) << 4;
    mn = (byte_at(w, 12 + g - 4) >> 4) | (byte_at(w, 8 + g - 4) >> 6) << 4;
  }
  const uint64_t dsc = dup2(__fmul_rn(d, (float)sc)), ndmn = dup2(-__fmul_rn(dmin, (float)mn));
  const uint64_t off = dup2(-8388608.0f);  // -2^23
  const int wq = 4 + 8 * (g >> 1);         // the group's 32 qs bytes: words wq .. wq + 7
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const uint32_t v = (g & 1) ? (w[wq + k] >> 4) & 0x0F0F0F0Fu : w[wq + k] & 0x0F0F0F0Fu;
    uint64_t a, b;
    magic4(v, a, b);
    o16[2 * k] = bf16x2(add2(mul2(add2(a, off), dsc), ndmn));
    o16[2 * k + 1] = bf16x2(add2(mul2(add2(b, off), dsc), ndmn));
  }
}

// Q5_K group g of the stage's super-block (176 bytes: d, dmin, the twelve scale bytes, qh[32], qs[128]): 32 values
// q (d sc_g) - dmin mn_g with q = nibble | bit g of qh[l] << 4 (the reference's q45_k<true>)
__device__ __forceinline__ void dq_q5_k_group(const uint32_t* w, int g, uint32_t* o16) {
  const float d = half_at(w, 0), dmin = half_at(w, 2);
  int sc, mn;
  if (g < 4) {
    sc = byte_at(w, 4 + g) & 63;
    mn = byte_at(w, 8 + g) & 63;
  } else {
    sc = (byte_at(w, 12 + g - 4) & 15) | (byte_at(w, 4 + g - 4) >> 6) << 4;
    mn = (byte_at(w, 12 + g - 4) >> 4) | (byte_at(w, 8 + g - 4) >> 6) << 4;
  }
  const uint64_t dsc = dup2(__fmul_rn(d, (float)sc)), ndmn = dup2(-__fmul_rn(dmin, (float)mn));
  const uint64_t off = dup2(-8388608.0f);  // -2^23
  const int wq = 12 + 8 * (g >> 1);        // the group's 32 qs bytes: words wq .. wq + 7 (qh: words 4 .. 11)
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const uint32_t nib = (g & 1) ? (w[wq + k] >> 4) & 0x0F0F0F0Fu : w[wq + k] & 0x0F0F0F0Fu;
    const uint32_t v = nib | (((w[4 + k] >> g) & 0x01010101u) << 4);
    uint64_t a, b;
    magic4(v, a, b);
    o16[2 * k] = bf16x2(add2(mul2(add2(a, off), dsc), ndmn));
    o16[2 * k + 1] = bf16x2(add2(mul2(add2(b, off), dsc), ndmn));
  }
}

// a 32-bit word at byte b (b + off even) of a Q6_K window (16-byte aligned shared memory)
__device__ __forceinline__ uint32_t q6_word(const uint8_t* win, int b) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(win + (b & ~3));
  return (b & 2) ? __funnelshift_r(w[0], w[1], 16) : w[0];
}

// Q6_K values 64 sub + 32 H .. + 31 of the super-block that starts at byte off of the window win (the reference's
// q6_k, dequant.cpp:83-101: value 128 h + 32 jj + l = (low nibble for jj < 2, else high, of ql[64 h + 32 (jj & 1) + l]
// | crumb jj of qh[32 h + l] << 4) - 32, times sc[8 h + 2 jj + (l >= 16)] d (fp32, rounded once each): here
// h = sub / 2, jj = 2 (sub & 1) + H
template <int H>
__device__ __forceinline__ void dq_q6_k_block(const uint8_t* win, int off, int sub, uint32_t (&o)[16]) {
  const int h2 = sub >> 1, jj = 2 * (sub & 1) + H;
  const uint32_t dw = q6_word(win, off + 208);
  const float d = __half2float(__ushort_as_half((unsigned short)(dw & 0xFFFFu)));
  const uint32_t scw = q6_word(win, off + 192 + 8 * h2 + 2 * jj);  // (sc[8 h + 2 jj], sc[8 h + 2 jj + 1])
  const int sc0 = (int)(int8_t)(scw & 0xFFu), sc1 = (int)(int8_t)((scw >> 8) & 0xFFu);
  const uint64_t s0 = dup2(__fmul_rn((float)sc0, d)), s1 = dup2(__fmul_rn((float)sc1, d));
  const uint64_t bias = dup2(-8388640.0f);  // -(2^23 + 32)
  const int qlb = off + 64 * h2 + 32 * H, qhb = off + 128 + 32 * h2;
  const int sh = (sub & 1) ? 4 : 0, ch = 2 * jj;
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const uint32_t ql = q6_word(win, qlb + 4 * k), qh = q6_word(win, qhb + 4 * k);
    const uint32_t v = ((ql >> sh) & 0x0F0F0F0Fu) | (((qh >> ch) & 0x03030303u) << 4);
    uint64_t a, b;
    magic4(v, a, b);
    const uint64_t sc = k < 4 ? s0 : s1;
    o[2 * k] = bf16x2(mul2(add2(a, bias), sc));
    o[2 * k + 1] = bf16x2(mul2(add2(b, bias), sc));
  }
}

// Q3_K values 64 sub + 32 H .. + 31 of the super-block that starts at byte off of the window win (the reference's
// q3_k, dequant.cpp:103-117): 32-group g = 2 sub + H = (n, j) = (g / 4, g % 4); its value i: q = crumb j of
// qs[32 n + i] | bit (4 n + j) of hmask[i] << 2, times a = d (scale - 32) of its 16-value sub-block 2 g + i / 16 (the
// 6-bit scale: low nibble of byte s, s < 8, or the high nibble of byte s - 8, top crumb from byte 8 + s % 4 at bit
// 2 (s / 4)), as (q - 4) a (fp32, each rounded once: exact)
template <int H>
__device__ __forceinline__ void dq_q3_k_block(const uint8_t* win, int off, int sub, uint32_t (&o)[16]) {
  const int g = 2 * sub + H, n = g >> 2, j = g & 3;
  const float d = __half2float(__ushort_as_half((unsigned short)(q6_word(win, off + 108) & 0xFFFFu)));
  float a[2];
#pragma unroll
  for (int u = 0; u < 2; u++) {
    const int sb = 2 * g + u;
    const int lo = sb < 8 ? win[off + 96 + sb] & 15 : win[off + 96 + sb - 8] >> 4;
    const int top = (win[off + 104 + (sb & 3)] >> (2 * (sb >> 2))) & 3;
    a[u] = __fmul_rn(d, (float)((lo | top << 4) - 32));
  }
  const uint64_t s0 = dup2(a[0]), s1 = dup2(a[1]);
  const uint64_t bias = dup2(-8388612.0f);  // -(2^23 + 4)
#pragma unroll
  for (int k = 0; k < 8; k++) {  // values 4k .. 4k + 3
    const uint32_t qs = q6_word(win, off + 32 + 32 * n + 4 * k), hm = q6_word(win, off + 4 * k);
    const uint32_t v = ((qs >> (2 * j)) & 0x03030303u) | (((hm >> (4 * n + j)) & 0x01010101u) << 2);
    uint64_t p0, p1;
    magic4(v, p0, p1);
    const uint64_t sc = k < 4 ? s0 : s1;
    o[2 * k] = bf16x2(mul2(add2(p0, bias), sc));
    o[2 * k + 1] = bf16x2(mul2(add2(p1, bias), sc));
  }
}

// the IQ4_NL / IQ4_XS code values (dequant.cpp:119, ggml's non-linear grid) + 128, as bytes: four code indices (bytes
// < 16) to four grid bytes by two byte permutes over the 16-entry table in four registers, picked per byte by bit 3
__device__ __forceinline__ uint32_t iq4_bytes(uint32_t idx) {
  constexpr uint32_t G0 = 0x3F2D1801u, G1 = 0x766A5D4Fu, G2 = 0xA6998D81u, G3 = 0xF1D9C5B5u;  // 1, 24, 45, ... 241
  const uint32_t x = idx & 0x07070707u;
  const uint32_t s = x | (x >> 4);                            // (byte 0: i0 | i1 << 4, byte 2: i2 | i3 << 4)
  const uint32_t sel = (s & 0xFFu) | ((s >> 8) & 0xFF00u);    // (the four indices & 7 as selector nibbles)
  const uint32_t lo = __byte_perm(G0, G1, sel), hi = __byte_perm(G2, G3, sel);
  const uint32_t m = ((idx >> 3) & 0x01010101u) * 0xFFu;
  return (lo & ~m) | (hi & m);
}

// IQ4_NL block at byte o of the stage's row bytes (dequant.cpp:121-126: Q4_0's layout): 32 values d grid[q]
__device__ __forceinline__ void dq_iq4_nl_block(const uint32_t* w, int o, uint32_t* o16) {
  const uint64_t d = dup2(half_at(w, o)), off = dup2(-8388736.0f);  // -(2^23 + 128)
  uint32_t q[4];
  words16(w, o + 2, q);
#pragma unroll
  for (int k = 0; k < 4; k++) {
    uint64_t a, b, c, e;
    magic4(iq4_bytes(q[k] & 0x0F0F0F0Fu), a, b);         // values 4k .. 4k + 3 (low nibbles)
    magic4(iq4_bytes((q[k] >> 4) & 0x0F0F0F0Fu), c, e);  // values 16 + 4k .. (high nibbles)
    o16[2 * k] = bf16x2(mul2(d, add2(a, off)));
    o16[2 * k + 1] = bf16x2(mul2(d, add2(b, off)));
    o16[8 + 2 * k] = bf16x2(mul2(d, add2(c, off)));
    o16[8 + 2 * k + 1] = bf16x2(mul2(d, add2(e, off)));
  }
}

// IQ4_XS values 64 sub + 32 H .. + 31 of the super-block at byte off of the window (dequant.cpp:128-140): 32-group
// g = 2 sub + H with ls = nibble (g % 2) of byte 4 + g / 2 | crumb g of the u16 at byte 2 << 4, w = (d (ls - 32)) grid[q]
// over its 16 code bytes at 8 + 16 g in Q4_0's order
template <int H>
__device__ __forceinline__ void dq_iq4_xs_block(const uint8_t* win, int off, int sub, uint32_t (&o)[16]) {
  const int g = 2 * sub + H;
  const uint32_t w0 = q6_word(win, off);  // (d, then the high scale crumbs)
  const float d = __half2float(__ushort_as_half((unsigned short)(w0 & 0xFFFFu)));
  const int ls = ((win[off + 4 + (g >> 1)] >> (4 * (g & 1))) & 15) | (int)((w0 >> (16 + 2 * g)) & 3u) << 4;
  const uint64_t dl = dup2(__fmul_rn(d, (float)(ls - 32))), bias = dup2(-8388736.0f);  // -(2^23 + 128)
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const uint32_t qw = q6_word(win, off + 8 + 16 * g + 4 * k);
    uint64_t a, b, c, e;
    magic4(iq4_bytes(qw & 0x0F0F0F0Fu), a, b);
    magic4(iq4_bytes((qw >> 4) & 0x0F0F0F0Fu), c, e);
    o[2 * k] = bf16x2(mul2(dl, add2(a, bias)));
    o[2 * k + 1] = bf16x2(mul2(dl, add2(b, bias)));
    o[8 + 2 * k] = bf16x2(mul2(dl, add2(c, bias)));
    o[8 + 2 * k + 1] = bf16x2(mul2(dl, add2(e, bias)));
  }
}

// the 16-byte chunks [lo, hi] of a row's stage bytes that block / group 2 sub + h of a 256-value chunk reads
template <int QT, int H>
struct BlockSpan {
  static constexpr int b(int sub) { return 2 * sub + H; }
  static constexpr int lo(int sub) {
    return QT == ARTLITE_Q4_0 || QT == ARTLITE_IQ4_NL ? (18 * b(sub)) / 16 : QT == ARTLITE_Q8_0 ? (34 * b(sub)) / 16
         : QT == ARTLITE_Q4_1 ? (20 * b(sub)) / 16 : 0;
  }
  static constexpr int hi(int sub) {
    return QT == ARTLITE_Q4_0 || QT == ARTLITE_IQ4_NL ? (18 * b(sub) + 17) / 16
         : QT == ARTLITE_Q4_1 ? (20 * b(sub) + 19) / 16
         : QT == ARTLITE_Q8_0 ? (34 * b(sub) + 33) / 16
         : QT == ARTLITE_Q4_K ? 0 : 2;  // (Q4_K: the header; Q5_K: the header and qh)
  }
  // Q4_K / Q5_K: the group's qs bytes (Q4_K 16 + 32 sub, Q5_K 48 + 32 sub): chunks qlo, qlo + 1
  static constexpr int qlo(int sub) { return QT == ARTLITE_Q4_K ? 1 + 2 * sub : 3 + 2 * sub; }
};

// block / group 2 sub + H of the stage row at src (its raw bytes, 16-byte chunks) as 16 bf16 pairs
template <int QT, int H>
__device__ __forceinline__ void dequant_block(const uint4* src, uint32_t* w, int sub, uint32_t (&o)[16]) {
  using S = BlockSpan<QT, H>;
#pragma unroll
  for (int v = S::lo(sub); v <= S::hi(sub); v++) {
    const uint4 u = src[v];
    w[4 * v] = u.x, w[4 * v + 1] = u.y, w[4 * v + 2] = u.z, w[4 * v + 3] = u.w;
  }
  if constexpr (QT == ARTLITE_Q4_K || QT == ARTLITE_Q5_K) {
#pragma unroll
    for (int v = S::qlo(sub); v <= S::qlo(sub) + 1; v++) {
      const uint4 u = src[v];
      w[4 * v] = u.x, w[4 * v + 1] = u.y, w[4 * v + 2] = u.z, w[4 * v + 3] = u.w;
    }
  }
  const int b = 2 * sub + H;
  if constexpr (QT == ARTLITE_Q4_0) dq_q4_0_block(w, 18 * b, o);
  else if constexpr (QT == ARTLITE_IQ4_NL) dq_iq4_nl_block(w, 18 * b, o);
  else if constexpr (QT == ARTLITE_Q4_1) dq_q4_1_block(w, 20 * b, o);
  else if constexpr (QT == ARTLITE_Q8_0) dq_q8_0_block(w, 34 * b, o);
  else if constexpr (QT == ARTLITE_Q5_K) dq_q5_k_group(w, b, o);
  else dq_q4_k_group(w, b, o);
}

// ---------------------------------------------------------------- the kernel

// the kernel's shared-memory pipeline depth: A + B stages and raw weight stages, per format and mode
__host__ __device__ constexpr int b_stage_bytes(bool pair) { return pair ? B_BYTES / 2 : B_BYTES; }
__host__ __device__ constexpr int ab_stages(int qt, bool pair) {
  return pair ? (qt == ARTLITE_Q8_0 || qt == ARTLITE_Q5_K || qt == ARTLITE_Q6_K || qt == ARTLITE_IQ4_XS ||
                         qt == ARTLITE_Q4_1
                     ? 4
                     : 5)
              : 3;
}
// the epilogue's transpose buffers: per epilogue warp 32 token rows of up to 32 bf16 values, rows 80 bytes apart
// (16-byte row reads of 8 consecutive lanes fall in distinct banks)
constexpr int kEpiRow = 80, kEpiWarp = 32 * kEpiRow;
__host__ __device__ constexpr size_t smem_bytes(int qt, bool pair) {
  return 1024 + (size_t)ab_stages(qt, pair) * (A_BYTES + b_stage_bytes(pair)) +
         (size_t)raw_stages(qt) * BM * raw_pitch(qt) + 4 * kEpiWarp + 512;
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// the shared::cluster address of this CTA's variable at p in cluster CTA `rank`
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// the pair's TMA load: the bytes land in this CTA, the transaction count goes to the barrier at `bar` (a
// shared::cluster address, here the leader CTA's)
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void mma_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(id), "r"(acc));
}
// MMA completion to the barrier at the same offset in both CTAs of the pair
__device__ __forceinline__ void commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}
// a wait whose barrier also receives the peer CTA's arrivals (acquire at cluster scope)
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool wait_cluster(int* abort, uint64_t* bar, uint32_t parity, DevStatus* st, int where) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  for (;;) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (*(volatile int*)abort) return false;
    if (clock64() - t0 > kWaitCycles) {
      *(volatile int*)abort = 1;
      report(st, ARTLITE_ETIMEOUT, where, (int)blockIdx.x, 0);
      return false;
    }
  }
}

// PAIR: a cluster of two CTAs on two SMs runs each tile as one M = 256 MMA (tcgen05 cta_group::2): each CTA
// dequantises its own 128 weight rows (A halves) and loads half of the tile's token rows (B halves, N / 2 each), the
// leader CTA issues the MMAs, whose completion is committed to both CTAs' barriers; each CTA's TMEM holds its 128
// rows of the accumulator and its epilogue writes them. Per SM the token rows come from L2 once per 256 weight rows
// instead of once per 128.
template <int QT, bool GU, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1) tc_expert_gemm(const __grid_constant__ Params p) {
  constexpr int CB = chunk_bytes(QT);
  constexpr int NW = CB / 4;
  constexpr int R = raw_stages(QT);
  constexpr int SS = ab_stages(QT, PAIR);
  constexpr int BB = b_stage_bytes(PAIR);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = base;
  uint8_t* sB = sA + SS * A_BYTES;
  uint8_t* sR = sB + SS * BB;
  constexpr int RPITCH = raw_pitch(QT);
  uint8_t* sE = sR + R * BM * RPITCH;  // the epilogue warps' transpose buffers
  Smem* sm = reinterpret_cast<Smem*>(sE + 4 * kEpiWarp);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total = p.toff[p.E];
  const uint32_t crank = PAIR ? cluster_rank() : 0;  // 0: the leader
  const int t0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int tstep = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  constexpr int NPEER = PAIR ? 2 : 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < SS; i++) {
      mbar_init(&sm->full_a[i], 256 * NPEER);
      mbar_init(&sm->full_b[i], 1);
      mbar_init(&sm->empty[i], 1);
    }
    for (int i = 0; i < R; i++) {
      mbar_init(&sm->raw_full[i], windowed(QT) ? 32 : 1);  // (Q6_K / Q3_K: the copy warp's lanes; else the TMA)
      mbar_init(&sm->raw_empty[i], 256);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&sm->tfull[i], 1);
      mbar_init(&sm->tempty[i], 128 * NPEER);
    }
    sm->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    if constexpr (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm->tmem_base)),
                   "r"(512));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm->tmem_base)),
                   "r"(512));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  fence_before();
  if constexpr (PAIR) cluster_sync();
  else __syncthreads();
  fence_after();
  const uint32_t tmem = sm->tmem_base;
  const int ksteps = p.K / BK;

  if (warp == 0 && lane == 0) {
    // ---------------- producer of the token rows (B stages; in a pair each CTA its half, counted by the leader)
    int s = 0, sph = 0;
    for (int t = t0; t < total; t += tstep) {
      const Tile T = tile_of(p, t);
      const int half = T.n_mma / 2;
      for (int ks = 0; ks < ksteps; ks++) {
        if (!wait(&sm->abort, &sm->empty[s], sph ^ 1, p.status, 2)) goto out;
        if constexpr (PAIR) {
          if (crank == 0) mbar_expect_tx(&sm->full_b[s], 2 * BB);
          tma_load_2d_pair(sB + s * BB, &p.map_x, peer_addr(&sm->full_b[s], 0), ks * BK,
                           (int)T.row0 + (int)crank * half);
        } else {
          mbar_expect_tx(&sm->full_b[s], BB);
          tma_load_2d(sB + s * BB, &p.map_x, &sm->full_b[s], ks * BK, (int)T.row0);
        }
        if (++s == SS) s = 0, sph ^= 1;
      }
    }
  } else if (warp == 0 && lane == 1 && !windowed(QT)) {
    // ---------------- producer of the raw weight rows (R stages of 256 values, ahead of the B stages)
    int r = 0, rph = 0;
    for (int t = t0; t < total; t += tstep) {
      const Tile T = tile_of(p, t);
      const int m = NPEER * T.m + (int)crank;  // this CTA's 64 features (gu) / 128 rows (down)
      for (int kc = 0; kc < p.K / KC; kc++) {
        if (!wait(&sm->abort, &sm->raw_empty[r], rph ^ 1, p.status, 1)) goto out;
        uint8_t* dst = sR + r * BM * CB;
        mbar_expect_tx(&sm->raw_full[r], BM * CB);
        if (GU) {
          const int row = T.we * p.N + 64 * m;
          tma_load_2d(dst, &p.map_w0, &sm->raw_full[r], kc * (CB / 2), row);
          tma_load_2d(dst + 64 * CB, &p.map_w1, &sm->raw_full[r], kc * (CB / 2), row);
        } else {
          tma_load_2d(dst, &p.map_w0, &sm->raw_full[r], kc * (CB / 2), T.we * p.N + BM * m);
        }
        if (++r == R) r = 0, rph ^= 1;
      }
    }
  } else if (warp == 1 && lane == 0 && crank == 0) {
    // ---------------- MMA issuer (the leader of a pair)
    int s = 0, sph = 0, acc = 0, aph = 0;
    for (int t = t0; t < total; t += tstep) {
      const Tile T = tile_of(p, t);
      if (!(PAIR ? wait_cluster(&sm->abort, &sm->tempty[acc], aph ^ 1, p.status, 3)
                 : wait(&sm->abort, &sm->tempty[acc], aph ^ 1, p.status, 3)))
        goto out;
      fence_after();
      const uint32_t id = idesc(PAIR ? 2 * BM : BM, T.n_mma);
      const uint32_t d = tmem + acc * BNMAX;
      for (int ks = 0; ks < ksteps; ks++) {
        if (!(PAIR ? wait_cluster(&sm->abort, &sm->full_a[s], sph, p.status, 4)
                   : wait(&sm->abort, &sm->full_a[s], sph, p.status, 4)))
          goto out;
        if (!(PAIR ? wait_cluster(&sm->abort, &sm->full_b[s], sph, p.status, 5)
                   : wait(&sm->abort, &sm->full_b[s], sph, p.status, 5)))
          goto out;
        fence_after();
        const uint64_t da = sdesc(smem_u32(sA + s * A_BYTES)), db = sdesc(smem_u32(sB + s * BB));
#pragma unroll
        for (int k = 0; k < BK / 16; k++) {
          if constexpr (PAIR) mma_pair(d, da + 2 * k, db + 2 * k, id, (ks | k) != 0);
          else mma(d, da + 2 * k, db + 2 * k, id, (ks | k) != 0);
        }
        if constexpr (PAIR) commit_pair(&sm->empty[s]);
        else commit(&sm->empty[s]);
        if (++s == SS) s = 0, sph ^= 1;
      }
      if constexpr (PAIR) commit_pair(&sm->tfull[acc]);
      else commit(&sm->tfull[acc]);
      if (++acc == 2) acc = 0, aph ^= 1;
    }
  } else if (warp >= 2 && warp < 10) {
    // ---------------- dequant: all eight warps on every step, in step order (as every other role waits on every phase
    // of the barriers it uses: a stage's writers never skip one of its phases). Thread (h, i), h = its warp's half
    // (warps 2-5: 0, 6-9: 1), i its A row, decodes values 32 h .. 32 h + 31 of each 64-value step of its row: one
    // 32-value block (Q4_0 / Q8_0) or group (Q4_K / Q5_K), from only that block's raw bytes.
    const int h = (warp - 2) >> 2, i = threadIdx.x - 64 - 128 * h;
    int raw_row = i;
    if (GU) {
      const int q = i >> 5, l = i & 31;
      raw_row = l < 16 ? 16 * q + l : 64 + 16 * q + (l - 16);
    }
    int n = 0, r = 0, rph = 0;  // n: the step counter shared with the producer and the MMA issuer
    const uint32_t full_a0 = PAIR ? peer_addr(&sm->full_a[0], 0) : 0;  // (the leader's barriers, for a peer's arrivals)
    for (int t = t0; t < total; t += tstep) {
      for (int kc = 0; kc < p.K / KC; kc++) {
        if (!wait(&sm->abort, &sm->raw_full[r], rph, p.status, 6)) goto out;
        const uint4* src = reinterpret_cast<const uint4*>(sR + r * BM * RPITCH + raw_row * RPITCH);
        int q6off = 0;  // (Q6_K / Q3_K: where the row's super-block starts in its window)
        if constexpr (windowed(QT)) q6off = (int)(raw_src<GU>(p, tile_of(p, t), NPEER, crank, raw_row, kc) & 15);
#pragma unroll
        for (int sub = 0; sub < KC / BK; sub++) {
          const int step = n + sub, s = step % SS;
          const uint32_t ph = (step / SS) & 1;
          uint32_t w[NW + 4];
          uint32_t o[16];
          const int blk = 2 * sub + h;  // (the 32-value block / group)
          if constexpr (QT == ARTLITE_Q6_K) {
            if (h == 0) dq_q6_k_block<0>(reinterpret_cast<const uint8_t*>(src), q6off, sub, o);
            else dq_q6_k_block<1>(reinterpret_cast<const uint8_t*>(src), q6off, sub, o);
          } else if constexpr (QT == ARTLITE_Q3_K) {
            if (h == 0) dq_q3_k_block<0>(reinterpret_cast<const uint8_t*>(src), q6off, sub, o);
            else dq_q3_k_block<1>(reinterpret_cast<const uint8_t*>(src), q6off, sub, o);
          } else if constexpr (QT == ARTLITE_IQ4_XS) {
            if (h == 0) dq_iq4_xs_block<0>(reinterpret_cast<const uint8_t*>(src), q6off, sub, o);
            else dq_iq4_xs_block<1>(reinterpret_cast<const uint8_t*>(src), q6off, sub, o);
          } else {
            if (h == 0) dequant_block<QT, 0>(src, w, sub, o);
            else dequant_block<QT, 1>(src, w, sub, o);
          }
          if (!wait(&sm->abort, &sm->empty[s], ph ^ 1, p.status, 7)) goto out;
          uint8_t* row = sA + s * A_BYTES + i * 128;
#pragma unroll
          for (int c = 0; c < 4; c++)
            *reinterpret_cast<uint4*>(row + (((4 * h + c) ^ (i & 7)) << 4)) =
                make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
          (void)blk;
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          if (PAIR && crank != 0) arrive_cluster(full_a0 + s * (uint32_t)sizeof(uint64_t));
          else mbar_arrive(&sm->full_a[s]);
        }
        mbar_arrive(&sm->raw_empty[r]);  // (every lane, after its last use of the stage's bytes)
        if (++r == R) r = 0, rph ^= 1;
        n += KC / BK;
      }
    }
  } else if (warp == 14) {
    // ---------------- Q6_K / Q3_K: the copy warp. Each lane copies four rows' windows (from the 16-byte boundary at or
    // below the row's super-block: 224 bytes for Q6_K, 128 for Q3_K) with 16-byte cp.async, then arrives on the stage's
    // full barrier when its copies have landed
    if constexpr (windowed(QT)) {
      int r = 0, rph = 0;
      for (int t = t0; t < total; t += tstep) {
        const Tile T = tile_of(p, t);
        for (int kc = 0; kc < p.K / KC; kc++) {
          if (!wait(&sm->abort, &sm->raw_empty[r], rph ^ 1, p.status, 1)) goto out;
          uint8_t* dst = sR + r * BM * RPITCH;
#pragma unroll
          for (int j = 0; j < BM / 32; j++) {
            const int row = lane + 32 * j;
            const uintptr_t g = raw_src<GU>(p, T, NPEER, crank, row, kc) & ~(uintptr_t)15;
            const uint32_t d0 = smem_u32(dst + row * RPITCH);
#pragma unroll
            for (int c = 0; c < window_chunks(QT); c++)
              asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d0 + 16 * c), "l"(g + 16 * c) : "memory");
          }
          asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&sm->raw_full[r])) : "memory");
          if (++r == R) r = 0, rph ^= 1;
        }
      }
      asm volatile("cp.async.wait_all;" ::: "memory");
    }
  } else if (warp >= 10) {
    // ---------------- epilogue: TMEM lanes 32 q .. 32 q + 31
    const int q = warp & 3;
    int acc = 0, aph = 0;
    const uint32_t tempty0 = PAIR ? peer_addr(&sm->tempty[0], 0) : 0;
    for (int t = t0; t < total; t += tstep) {
      Tile T = tile_of(p, t);
      T.m = NPEER * T.m + (int)crank;  // this CTA's rows
      if (!wait(&sm->abort, &sm->tfull[acc], aph, p.status, 8)) goto out;
      fence_after();
      // 32 columns at a time, the next chunk's TMEM load in flight while this chunk is stored
      const uint32_t base = tmem + ((uint32_t)(32 * q) << 16) + acc * BNMAX;
      const int nch = (T.n_mma + 31) / 32;
      // a 32-token chunk: values into this warp's buffer as [token][column] bf16, then each lane stores its token's
      // columns with 16-byte stores (gu: 16 features, 32 B; down: 32 rows, 64 B of the output row)
      uint8_t* eb = sE + q * kEpiWarp;
      auto emit = [&](const uint32_t(&v)[32], int c0) {
        if (GU) {
          const bool gate = lane < 16;
#pragma unroll
          for (int j = 0; j < 16; j++) {
            const float mine = __uint_as_float(gate ? v[j] : v[16 + j]);
            const float send = __uint_as_float(gate ? v[16 + j] : v[j]);
            const float other = __shfl_xor_sync(0xFFFFFFFFu, send, 16);
            const float g = gate ? mine : other, u = gate ? other : mine;
            const float h = __fdividef(g, 1.0f + __expf(-g)) * u;
            const int tok = j + (gate ? 0 : 16);  // (within the chunk)
            *reinterpret_cast<uint16_t*>(eb + tok * kEpiRow + 2 * (lane & 15)) = __bfloat16_as_ushort(__float2bfloat16_rn(h));
          }
          __syncwarp();
          const int tok = c0 + lane;
          if (tok < T.valid) {
            const uint4* src = reinterpret_cast<const uint4*>(eb + lane * kEpiRow);
            uint4* dst = reinterpret_cast<uint4*>(p.out + (T.row0 + tok) * p.N + 64 * T.m + 16 * q);
            dst[0] = src[0];
            dst[1] = src[1];
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; j++)
            *reinterpret_cast<uint16_t*>(eb + j * kEpiRow + 2 * lane) = __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(v[j])));
          __syncwarp();
          const int tok = c0 + lane;
          if (tok < T.valid) {
            const uint4* src = reinterpret_cast<const uint4*>(eb + lane * kEpiRow);
            uint4* dst = reinterpret_cast<uint4*>(p.out + (T.row0 + tok) * p.N + BM * T.m + 32 * q);
#pragma unroll
            for (int c = 0; c < 4; c++) dst[c] = src[c];
          }
        }
        __syncwarp();  // (the buffer is free for the next chunk)
      };
      uint32_t va[32], vb[32];
      tmem_ld32(base, va);
      tmem_wait32(va);
      for (int c = 0; c < nch; c += 2) {
        if (c + 1 < nch) tmem_ld32(base + 32 * (c + 1), vb);
        emit(va, 32 * c);
        if (c + 1 < nch) {
          tmem_wait32(vb);
          if (c + 2 < nch) tmem_ld32(base + 32 * (c + 2), va);
          emit(vb, 32 * (c + 1));
          if (c + 2 < nch) tmem_wait32(va);
        }
      }
      fence_before();
      if (PAIR && crank != 0) arrive_cluster(tempty0 + acc * (uint32_t)sizeof(uint64_t));
      else mbar_arrive(&sm->tempty[acc]);
      if (++acc == 2) acc = 0, aph ^= 1;
    }
  }
out:
  __syncwarp();
  __syncthreads();
  if (*(volatile int*)&sm->abort && threadIdx.x == 0) {  // let issued copies and MMAs land before TMEM is freed
    const long long t0 = clock64();
    while (clock64() - t0 < 20000000LL) {
    }
  }
  if constexpr (PAIR) cluster_sync();  // (the leader's MMAs read the peer's shared memory until here)
  else __syncthreads();
  if (warp == 0) {
    fence_after();
    if constexpr (PAIR) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    else asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

}  // namespace tc

// ---------------------------------------------------------------- the router on the tensor cores
//
// logits (T x E fp32) = x (T x H bf16) . W_r^T, with W_r (fp32) split into three bf16 planes hi + mid + lo
// (hi = bf16(w), mid = bf16(w - hi), lo = bf16(w - hi - mid): |w - (hi + mid + lo)| <= 2^-24 |w|); every product of a
// bf16 x with a plane is exact in fp32 and the three MMAs accumulate into one fp32 accumulator: the fp32 GEMM's logits
// to within fp32 rounding of the sums. Per tile 128 experts (A: the planes, TMA, 128-byte swizzle) x 128 tokens (B),
// K in stages of 64 (each stage the three planes and the token rows). Warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
// (logits[t, e] + bias[e], fp32, coalesced over e).
namespace rt {
constexpr int BM = 128, BN = 128, BK = 64, S = 3, PLANES = 3;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE = PLANES * A_BYTES + B_BYTES;
constexpr int kThreads = 192;

struct Params {
  CUtensorMap map_w, map_x;  // w: the planes stacked (PLANES E rows of H), x: T rows of H
  const float* bias;
  float* logits;
  DevStatus* status;
  int64_t T;
  int E, H, planes;
};

struct Smem {
  uint64_t full[S], empty[S], tfull;
  uint32_t tmem_base;
  int abort;
};
}  // namespace rt

__global__ void __launch_bounds__(rt::kThreads, 1) router_tc_kernel(const __grid_constant__ rt::Params p) {
  using namespace rt;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  rt::Smem* sm = reinterpret_cast<rt::Smem*>(base + S * STAGE);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mtiles = p.E / BM;
  const int tile_t = blockIdx.x / mtiles, tile_m = blockIdx.x % mtiles;
  const int64_t t0 = (int64_t)tile_t * BN;
  const int valid = (int)min64((int64_t)BN, p.T - t0);
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; i++) {
      tc::mbar_init(&sm->full[i], 1);
      tc::mbar_init(&sm->empty[i], 1);
    }
    tc::mbar_init(&sm->tfull, 1);
    sm->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::smem_u32(&sm->tmem_base)),
                 "r"(128));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = sm->tmem_base;
  const int ksteps = p.H / BK;
  if (warp == 0 && lane == 0) {
    int s = 0, ph = 0;
    for (int ks = 0; ks < ksteps; ks++) {
      if (!tc::wait(&sm->abort, &sm->empty[s], ph ^ 1, p.status, 21)) goto out;
      uint8_t* st = base + s * STAGE;
      tc::mbar_expect_tx(&sm->full[s], p.planes * A_BYTES + B_BYTES);
      for (int pl = 0; pl < p.planes; pl++)
        tc::tma_load_2d(st + pl * A_BYTES, &p.map_w, &sm->full[s], ks * BK, pl * p.E + tile_m * BM);
      tc::tma_load_2d(st + PLANES * A_BYTES, &p.map_x, &sm->full[s], ks * BK, (int)t0);
      if (++s == S) s = 0, ph ^= 1;
    }
  } else if (warp == 1 && lane == 0) {
    int s = 0, ph = 0;
    const uint32_t id = tc::idesc(BM, BN);
    for (int ks = 0; ks < ksteps; ks++) {
      if (!tc::wait(&sm->abort, &sm->full[s], ph, p.status, 22)) goto out;
      tc::fence_after();
      uint8_t* st = base + s * STAGE;
      const uint64_t db = tc::sdesc(tc::smem_u32(st + PLANES * A_BYTES));
      for (int pl = 0; pl < p.planes; pl++) {
        const uint64_t da = tc::sdesc(tc::smem_u32(st + pl * A_BYTES));
#pragma unroll
        for (int k = 0; k < BK / 16; k++) tc::mma(tmem, da + 2 * k, db + 2 * k, id, (ks | pl | k) != 0);
      }
      tc::commit(&sm->empty[s]);
      if (++s == S) s = 0, ph ^= 1;
    }
    tc::commit(&sm->tfull);
  } else if (warp >= 2) {
    const int q = warp & 3;
    if (!tc::wait(&sm->abort, &sm->tfull, 0, p.status, 23)) goto out;
    tc::fence_after();
    const int e = tile_m * BM + 32 * q + lane;
    const float b = p.bias ? p.bias[e] : 0.0f;
    for (int c0 = 0; c0 < BN; c0 += 32) {
      uint32_t v[32];
      tc::tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + c0, v);
      tc::tmem_wait32(v);
#pragma unroll
      for (int j = 0; j < 32; j++)
        if (c0 + j < valid) p.logits[(t0 + c0 + j) * p.E + e] = __uint_as_float(v[j]) + b;
    }
    tc::fence_before();
  }
out:
  __syncwarp();
  __syncthreads();
  if (*(volatile int*)&sm->abort && threadIdx.x == 0) {
    const long long c = clock64();
    while (clock64() - c < 20000000LL) {
    }
  }
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(128));
  }
}

// W_r (E x H, fp32 or bf16) -> the bf16 planes (planes x E x H): fp32 into hi, mid, lo; bf16 copied as one plane
__global__ void router_split_kernel(const void* w, int w_dtype, int64_t n, uint16_t* planes) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  if (w_dtype == ARTLITE_BF16) {
    planes[i] = reinterpret_cast<const uint16_t*>(w)[i];
    return;
  }
  const float v = reinterpret_cast<const float*>(w)[i];
  const __nv_bfloat16 hi = __float2bfloat16_rn(v);
  const float r1 = __fsub_rn(v, __bfloat162float(hi));
  const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
  const float r2 = __fsub_rn(r1, __bfloat162float(mid));
  planes[i] = __bfloat16_as_ushort(hi);
  planes[n + i] = __bfloat16_as_ushort(mid);
  planes[2 * n + i] = __bfloat16_as_ushort(__float2bfloat16_rn(r2));
}

// ---------------------------------------------------------------- host side

namespace {

typedef CUresult (*EncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
  static EncodeTiled fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  }
  return fn;
}

// a 2D map over rows x row_bytes of 16-bit elements (raw GGUF bytes or bf16 values)
int make_map(CUtensorMap* m, const void* base, int64_t row_elems, int64_t rows, int box_x, int box_y, bool swizzle) {
  EncodeTiled enc = encode_fn();
  AL_CHECK(enc, ARTLITE_ECUDA, "tc gemm: cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)row_elems, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(row_elems * 2)};
  const cuuint32_t box[2] = {(cuuint32_t)box_x, (cuuint32_t)box_y};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, swizzle ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 2,
                         const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  AL_CHECK(r == CUDA_SUCCESS, ARTLITE_ECUDA, "tc gemm: cuTensorMapEncodeTiled failed (%d): %lld x %lld box %d x %d",
           (int)r, (long long)row_elems, (long long)rows, box_x, box_y);
  return ARTLITE_OK;
}

}  // namespace

int make_raw_map(CUtensorMap* m, const void* base, int64_t row_bytes, int64_t rows, int box_bytes, int box_rows) {
  return make_map(m, base, row_bytes / 2, rows, box_bytes / 2, box_rows, false);
}

bool router_tc_supported(int E, int H, int x_dtype) {
  return x_dtype == ARTLITE_BF16 && E % rt::BM == 0 && H % rt::BK == 0;
}

int router_split(const void* w, int w_dtype, int E, int H, uint16_t* planes, cudaStream_t st) {
  const int64_t n = (int64_t)E * H;
  router_split_kernel<<<(unsigned)cdiv(n, 256), 256, 0, st>>>(w, w_dtype, n, planes);
  AL_LAUNCHED();
  return ARTLITE_OK;
}

int launch_router_tc(const uint16_t* x, const uint16_t* planes, int n_planes, const float* bias, int64_t T, int H,
                     int E, int64_t x_rows, float* logits, DevStatus* status, cudaStream_t st) {
  AL_CHECK(router_tc_supported(E, H, ARTLITE_BF16) && n_planes >= 1 && n_planes <= rt::PLANES, ARTLITE_EUNSUPPORTED,
           "router tc: E %d H %d planes %d", E, H, n_planes);
  AL_CHECK(((uintptr_t)x % 16) == 0 && ((uintptr_t)planes % 16) == 0, ARTLITE_EINVAL, "router tc: unaligned operand");
  if (T == 0) return ARTLITE_OK;
  rt::Params p{};
  AL_TRY(make_map(&p.map_w, planes, H, (int64_t)n_planes * E, rt::BK, rt::BM, true));
  AL_TRY(make_map(&p.map_x, x, H, x_rows, rt::BK, rt::BN, true));
  p.bias = bias;
  p.logits = logits;
  p.status = status;
  p.T = T;
  p.E = E;
  p.H = H;
  p.planes = n_planes;
  const size_t smem = 1024 + rt::S * rt::STAGE + sizeof(rt::Smem) + 64;
  AL_CUDA(cudaFuncSetAttribute(router_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const unsigned grid = (unsigned)(cdiv(T, rt::BN) * (E / rt::BM));
  router_tc_kernel<<<grid, rt::kThreads, smem, st>>>(p);
  AL_LAUNCHED();
  return ARTLITE_OK;
}

bool tc_supported(int qtype, int K, int N) {
  return tc::chunk_bytes(qtype) > 0 && K % tc::KC == 0 && N % tc::BM == 0;
}

size_t tc_sched_bytes(int E) { return sizeof(int32_t) * (E + 1); }

// the pair (cta_group::2) kernel where the shape splits into pairs (ARTLITE_TC_PAIR=0: the one-CTA kernel): it halves
// each SM's token-operand traffic (measured at T = 16384, Q4_0: gate/up 1.08 -> 1.01 ms, down 0.60 -> 0.55 ms)
bool tc_use_pair(int N, bool gu) {
  const char* v = getenv("ARTLITE_TC_PAIR");  // (read per launch: a caller may switch it between forwards)
  const bool off = v && v[0] == '0';
  return !off && (gu ? N % 128 == 0 : N % 256 == 0);
}

int launch_tc_gemm(const TcGemmArgs& a, bool gu, cudaStream_t st) {
  AL_CHECK(tc_supported(a.qtype, a.K, a.N), ARTLITE_EUNSUPPORTED, "tc gemm: type %d K %d N %d", a.qtype, a.K, a.N);
  // (Q6_K rows need not be 16-byte pitched: the copy warp reads 16-byte-aligned windows; the TMA formats' rows must be)
  AL_CHECK((tc::windowed(a.qtype) || a.row_bytes % 16 == 0) &&
               a.row_bytes == (int64_t)a.K / tc::KC * tc::chunk_bytes(a.qtype), ARTLITE_EINVAL,
           "tc gemm: row bytes %lld", (long long)a.row_bytes);
  AL_CHECK(((uintptr_t)a.w0 % 16) == 0 && (!gu || ((uintptr_t)a.w1 % 16) == 0) && ((uintptr_t)a.x % 16) == 0,
           ARTLITE_EINVAL, "tc gemm: unaligned operand");
  AL_CHECK(a.x_rows >= a.P + tc::BNMAX, ARTLITE_EINVAL, "tc gemm: x holds %lld rows, needs %lld", (long long)a.x_rows,
           (long long)(a.P + tc::BNMAX));
  if (a.P == 0) return ARTLITE_OK;
  const bool pair = tc_use_pair(a.N, gu);
  const int MT = (gu ? a.N / 64 : a.N / tc::BM) / (pair ? 2 : 1);  // tiles of weight rows per token tile
  tc::Params p{};
  const int cb = tc::chunk_bytes(a.qtype);
  const int64_t wrows = (int64_t)(a.wE > 0 ? a.wE : a.E) * a.N;
  if (!tc::windowed(a.qtype)) {
    AL_TRY(make_map(&p.map_w0, a.w0, a.row_bytes / 2, wrows, cb / 2, gu ? 64 : tc::BM, false));
    if (gu) AL_TRY(make_map(&p.map_w1, a.w1, a.row_bytes / 2, wrows, cb / 2, 64, false));
    else p.map_w1 = p.map_w0;
  }
  p.gw0 = static_cast<const uint8_t*>(a.w0);
  p.gw1 = static_cast<const uint8_t*>(gu ? a.w1 : a.w0);
  p.rb = a.row_bytes;
  p.cb = cb;
  AL_TRY(make_map(&p.map_x, a.x, a.K, a.x_rows, tc::BK, pair ? tc::BNMAX / 2 : tc::BNMAX, true));
  AL_TRY(launch_unit_scan(a.counts, a.E, tc::BNMAX, MT, static_cast<int32_t*>(a.sched), st));
  p.offsets = a.offsets;
  p.wexp = a.wexp;
  p.toff = static_cast<const int32_t*>(a.sched);
  p.out = a.out;
  p.status = a.status;
  p.E = a.E;
  p.K = a.K;
  p.N = a.N;
  p.MT = MT;
  const size_t smem = tc::smem_bytes(a.qtype, pair);
  int dev, sms;
  AL_CUDA(cudaGetDevice(&dev));
  AL_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  auto go = [&](auto kern) -> int {
    AL_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    if (pair) {
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = dim3((unsigned)(sms & ~1));
      cfg.blockDim = dim3(tc::kThreads);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = st;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      AL_CUDA(cudaLaunchKernelEx(&cfg, kern, p));
    } else {
      kern<<<sms, tc::kThreads, smem, st>>>(p);
    }
    AL_LAUNCHED();
    return ARTLITE_OK;
  };
#define AL_TC_CASE(QT)                                                                              \
  case QT:                                                                                          \
    return pair ? (gu ? go(tc::tc_expert_gemm<QT, true, true>) : go(tc::tc_expert_gemm<QT, false, true>)) \
                : (gu ? go(tc::tc_expert_gemm<QT, true, false>) : go(tc::tc_expert_gemm<QT, false, false>));
  switch (a.qtype) {
    AL_TC_CASE(ARTLITE_Q4_0)
    AL_TC_CASE(ARTLITE_Q8_0)
    AL_TC_CASE(ARTLITE_Q4_K)
    AL_TC_CASE(ARTLITE_Q5_K)
    AL_TC_CASE(ARTLITE_Q6_K)
    AL_TC_CASE(ARTLITE_Q3_K)
    AL_TC_CASE(ARTLITE_IQ4_NL)
    AL_TC_CASE(ARTLITE_Q4_1)
    AL_TC_CASE(ARTLITE_IQ4_XS)
    default: break;
  }
#undef AL_TC_CASE
  set_error("tc gemm: type %d", a.qtype);
  return ARTLITE_EUNSUPPORTED;
}

}  // namespace artlite
