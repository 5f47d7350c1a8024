// Blackwell (sm_100a) building blocks in inline PTX: mbarriers with bounded waits,
// TMA tiled and bulk copies, tcgen05 TMEM allocation, MMA, commit and loads.
//
// Descriptor layouts (PTX ISA, tcgen05 "Shared memory descriptor" and "Instruction
// descriptor"; the same bit fields as CUTLASS's cute/arch/mma_sm100_desc.hpp):
//   smem descriptor: start address >> 4 [0,14), leading byte offset >> 4 [16,30),
//                    stride byte offset >> 4 [32,46), version 1 [46,48), base offset
//                    [49,52), layout type [61,64) (2 = SWIZZLE_128B).
//   instr descriptor: c format [4,6) (1 F32, 2 S32), a format [7,10), b format [10,13)
//                    (f16 kind: 0 F16; i8 kind: 0 unsigned, 1 signed), a/b major
//                    [15], [16] (0 K-major), N >> 3 [17,23), M >> 4 [24,29).
#pragma once

#include <cstdint>

namespace crec {

// Wait limits: every wait gives up after kWaitNs of the global timer (or kSpinLimit polls, a
// backstop), records an error word and lets the kernel run to its end instead of hanging.
constexpr uint32_t kSpinLimit = 1u << 26;
constexpr uint64_t kWaitNs = 2000000000ull;

enum DeviceError : int {
  kErrNone = 0,
  kErrTimeoutFull = 1,
  kErrTimeoutEmpty = 2,
  kErrTimeoutTmemFull = 3,
  kErrTimeoutTmemEmpty = 4,
  kErrBadShape = 5,
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// A thread whose phase is not complete is suspended (issuing nothing) until it completes or
// kSuspendNs pass: waiting warps leave their sub-partition's issue slots to the warps that work.
constexpr uint32_t kSuspendNs = 1000000;

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits for the phase of `parity` to complete, at most limit_ns.  False on a timeout, after
// recording `code` in *err (the first error wins).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code,
                                          uint64_t limit_ns = kWaitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 15) == 0 && global_ns() - t0 > limit_ns) break;
  }
  if (err) atomicCAS(err, 0, code);
  return false;
}

// x / d by a multiply-high: magic = div_magic(d) = floor(2^32 / d) + 1 (d >= 2); exact whenever
// x * d < 2^32 (the error of magic * d over 2^32 is at most d).  d = 1 passes x through.
__host__ __device__ inline uint32_t div_magic(uint32_t d) {
  return d <= 1 ? 0u : static_cast<uint32_t>(0x100000000ull / d + 1);
}
__device__ __forceinline__ int fast_div(int x, int d, uint32_t magic) {
  return d <= 1 ? x : static_cast<int>(__umulhi(static_cast<uint32_t>(x), magic));
}

// One lane of a converged warp (the same lane each call while the whole warp is active).
__device__ __forceinline__ bool elect_one() {
  uint32_t e;
  asm volatile("{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}\n" : "=r"(e));
  return e != 0;
}

// mbar_wait by every lane of a converged warp; the vote makes the result warp-uniform, so a
// loop that leaves on a timeout keeps its counters uniform (and the MMA and TMA operands
// derived from them in uniform registers).
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, int* err, int code,
                                               uint64_t limit_ns = kWaitNs) {
  if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, err, code, limit_ns));
}

// TMA: a tiled box of a 3-d tensor map into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, int c0, int c1, int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// TMA: a tiled box of a 4-d tensor map into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_4d(void* dst, const void* tmap, int c0, int c1, int c2, int c3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

// Bulk copy of `bytes` (a multiple of 16, both ends 16-byte aligned) global -> shared.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Asynchronous prefetch of `bytes` (a multiple of 16, the start 16-byte aligned) of global memory
// into L2 by the bulk-copy unit; the issuing thread does not wait for it.
__device__ __forceinline__ void l2_prefetch_bulk(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---------------------------------------------------------------- tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand in the 128-byte swizzle: rows of 128 bytes, 8-row atoms 1024 bytes apart.
// `addr` is the shared address of the operand's first byte for this K step (the tile's base,
// 1024-aligned, plus the step's byte offset within the 128-byte row).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;            // leading byte offset (unused by K-major swizzled)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;    // stride byte offset: 8 rows x 128 bytes
  d |= static_cast<uint64_t>(1u) << 46;            // version (sm_100)
  d |= static_cast<uint64_t>(2u) << 61;            // SWIZZLE_128B
  return d;
}

// K-major operand in the 64- or 32-byte swizzle (layout types 4 and 6 of the descriptor's 3-bit
// field; 2 is the 128-byte one): rows of `row` bytes (64 or 32), 8-row atoms 8 * row bytes apart.
__device__ __forceinline__ uint64_t umma_desc_narrow(uint32_t addr, uint32_t row) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;                     // leading byte offset (unused by K-major swizzled)
  d |= static_cast<uint64_t>(((8u * row) >> 4) & 0x3FFFu) << 32;  // stride byte offset: 8 rows
  d |= static_cast<uint64_t>(1u) << 46;                     // version (sm_100)
  d |= static_cast<uint64_t>(row == 64 ? 4u : 6u) << 61;    // SWIZZLE_64B or SWIZZLE_32B
  return d;
}

// K-major operand without swizzle: 8-row core matrices of 16 bytes (128 contiguous bytes each);
// `lbo` the byte step between core matrices along K, `sbo` along M (or N) -- checked on the GPU
// against a host product, both ways round (only this reading gives it).
__device__ __forceinline__ uint64_t umma_desc_none(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;  // version (sm_100); layout type 0: no swizzle
  return d;
}

// Instruction descriptors, M = 128, both operands K-major.
__host__ __device__ constexpr uint32_t idesc_i8(int n) {  // A unsigned 8-bit, B signed 8-bit, D s32
  return (2u << 4) | (0u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) | ((128u >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_f16(int n) {  // A, B f16, D f32
  return (1u << 4) | (0u << 7) | (0u << 10) | (static_cast<uint32_t>(n >> 3) << 17) | ((128u >> 4) << 24);
}

template <bool kInt8>
__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  if constexpr (kInt8) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(
            d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
  } else {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
            d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
  }
}

// Arrives on `bar` once every MMA this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 consecutive 32-bit columns of this warp's 32 TMEM lanes: thread t gets lane (taddr's lane + t).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 16 consecutive columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Pins registers a tcgen05.ld wrote after the tcgen05.wait::ld that made them valid: the compiler
// sees the load's outputs as ready at the load, so without this it could move their uses above
// the wait.
template <int N>
__device__ __forceinline__ void tmem_pin(uint32_t (&r)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i])::"memory");
}

// A barrier among `count` threads of the block (a multiple of 32), id 1..15; id 0 is __syncthreads.
__device__ __forceinline__ void named_bar(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Exact integer <-> float conversions on the FMA and integer pipes instead of the conversion
// unit.  The floats in [2^23, 2^24) are the integers, one apart, so for an integer |s| < 2^22 the
// float with bits kMagicBits + s is kMagic + s exactly, and for a float |x| <= 2^22 the sum
// x + kMagic rounded to nearest (ties to even; kMagic is even) has bits kMagicBits + rint(x).
constexpr int32_t kMagicBits = 0x4B400000;
constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23

// s (|s| < 2^22) as a float, given s + kMagicBits.
__device__ __forceinline__ float magic_to_float(int32_t biased) { return __fsub_rn(__int_as_float(biased), kMagic); }
// rint(x) + kMagicBits for |x| <= 2^22 (round to nearest, ties to even, as __float2int_rn).
__device__ __forceinline__ int32_t magic_rint_bits(float x) { return __float_as_int(__fadd_rn(x, kMagic)); }

// Packed FP32 pairs (PTX add.rn.f32x2, sm_100): each half rounded to nearest even on its own,
// the same bits as __fadd_rn on each half (checked on 2^33 random pairs and on exact ties: no
// difference), one instruction for two.  Only the adds are packed: a packed product
// (mul.rn.f32x2) whose one use is a packed add is fused with it into one fused multiply-add by the
// assembler, despite the explicit rounding (measured: a quarter of such chains lose the product's
// rounding), while products from the scalar pipe feeding a packed add keep both roundings
// (measured: none differ).  So every product here is a __fmul_rn.
__device__ __forceinline__ float2 fadd2_rn(float2 a, float2 b) {
  float2 d;
  asm("{\n .reg .b64 a, b, d;\n mov.b64 a, {%2, %3};\n mov.b64 b, {%4, %5};\n add.rn.f32x2 d, a, b;\n"
      " mov.b64 {%0, %1}, d;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 fmul_pair_rn(float2 a, float2 b) {
  return make_float2(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y));
}
// Two biased sums (s + kMagicBits each, |s| < 2^22) as floats.
__device__ __forceinline__ float2 magic_to_float2(int32_t b0, int32_t b1) {
  return fadd2_rn(make_float2(__int_as_float(b0), __int_as_float(b1)), make_float2(-kMagic, -kMagic));
}
// The INT8 output stage of two sums (given biased, + kMagicBits) up to the code's rounding:
// (s * scale + bias) * inv_scale, each operation rounded on its own (the reference's
// epilogue_scalar, carbon/src/cpu/kernels.h:354-380, without residual or ReLU).
__device__ __forceinline__ float2 out_stage2(int32_t b0, int32_t b1, float2 scale, float2 bias, float inv) {
  return fmul_pair_rn(fadd2_rn(fmul_pair_rn(magic_to_float2(b0, b1), scale), bias), make_float2(inv, inv));
}
// float(s) rounded to nearest even for any int32 s, both halves, without the conversion unit:
// s = hi + lo with lo = s & 0xfff and hi = (s >> 12) * 4096; both are exact floats (lo below 2^12,
// hi / 4096 below 2^19 in magnitude, through kMagic), so their one rounded sum is float(s).
__device__ __forceinline__ float2 exact_i2f2(int32_t s0, int32_t s1) {
  const float2 hi = fmul_pair_rn(magic_to_float2(kMagicBits + (s0 >> 12), kMagicBits + (s1 >> 12)), make_float2(4096.0f, 4096.0f));
  const float2 lo = magic_to_float2((s0 & 0xfff) | kMagicBits, (s1 & 0xfff) | kMagicBits);
  return fadd2_rn(hi, lo);
}
// rint of both halves + kMagicBits (|x| <= 2^22).
__device__ __forceinline__ void magic_rint_bits2(float2 x, int32_t& r0, int32_t& r1) {
  const float2 t = fadd2_rn(x, make_float2(kMagic, kMagic));
  r0 = __float_as_int(t.x);
  r1 = __float_as_int(t.y);
}

// 32 bytes to global memory in one store (sm_100's 256-bit st.global; p 32-byte aligned).
__device__ __forceinline__ void st_global_v8(void* p, uint4 a, uint4 b) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(a.x), "r"(a.y), "r"(a.z),
               "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
               : "memory");
}

// Bytes hi and lo, each saturated to [0, 255], above them the low 16 bits of `upper`:
// upper << 16 | sat(hi) << 8 | sat(lo) (PTX cvt.pack.sat.u8.s32.b32).
__device__ __forceinline__ uint32_t pack_sat_u8x2(int32_t hi, int32_t lo, uint32_t upper) {
  uint32_t d;
  asm("cvt.pack.sat.u8.s32.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(hi), "r"(lo), "r"(upper));
  return d;
}
// Four codes as bytes (c[0] lowest), each saturated to [0, 255].
__device__ __forceinline__ uint32_t pack_sat_u8x4(const int32_t* c) {
  return pack_sat_u8x2(c[1], c[0], pack_sat_u8x2(c[3], c[2], 0u));
}

// 2^x, the hardware approximation (PTX ex2.approx.ftz.f32); 2^-inf = 0.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t elect_one_sync() {
  uint32_t pred = 0;
  asm volatile(
      "{\n .reg .b32 rx;\n .reg .pred px;\n elect.sync rx|px, %1;\n selp.b32 %0, 1, 0, px;\n}\n"
      : "=r"(pred)
      : "r"(0xffffffffu));
  return pred;
}

}  // namespace crec
