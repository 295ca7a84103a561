// Device helpers shared by the tensor-core prefill kernels (prefill.cu, head_dim 128; prefill_wide.cu, head_dim
// 512): the A-from-TMEM MMA, TMEM loads and stores of one lane's columns, the softmax's packed f32x2 arithmetic, an
// FMA-pipe exponential, bf16 packing and a barrier that ORs a predicate over its threads.
#pragma once

#include "common.cuh"
#include "tc.cuh"

namespace omni {
namespace pfx {

// D (TMEM) = A (TMEM) x B (smem) [+ D]; issued by one thread.
OMNI_DEV void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

OMNI_DEV void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 columns of this thread's lane without waiting (complete after tmem_wait_ld()).
OMNI_DEV void tmem_ld32_async(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// 2^x on the FMA and integer pipes, for x <= 127 (the softmax's arguments are at most 8): x = j + f with j the
// nearest integer (the 1.5 * 2^23 addition leaves j in the low mantissa bits of t) and f in [-0.5, 0.5]; 2^f from a
// cubic fitted here for relative error on [-0.5, 0.5] (7.5e-5 at most, far below bf16's 2^-9); 2^j added to the
// exponent field. x is clamped to -126 (2^-126 or a denormal below it: zero to a probability), so that the exponent
// field never wraps. Used for part of the probabilities, so that the special-function unit, which forms the others
// with ex2, is not the only pipe the exponentials load.
OMNI_DEV float ex2_fma(float x) {
  x = fmaxf(x, -126.f);
  const float t = x + 12582912.f;
  const float f = x - (t - 12582912.f);
  const float q = fmaf(fmaf(fmaf(0.055174146f, f, 0.24261758f), f, 0.69326109f), f, 0.99992758f);
  return __uint_as_float(__float_as_uint(q) + (__float_as_uint(t) << 23));
}

// Packed pairs of floats for the f32x2 forms of fma / add (one instruction for two elements on the FMA pipe).
OMNI_DEV uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
OMNI_DEV void f2_unpack(uint64_t v, float& lo, float& hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
OMNI_DEV uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
OMNI_DEV uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
OMNI_DEV float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Two floats rounded to bf16 and packed (lo in the low half).
OMNI_DEV uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

OMNI_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

OMNI_DEV void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

OMNI_DEV void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

OMNI_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

OMNI_DEV bool sync_or(int id, int count, bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "barrier.cta.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(out)
      : "r"((uint32_t)pred), "r"(id), "r"(count)
      : "memory");
  return out != 0;
}

// Unit u -> (b, h, qt). The (row, head) pairs are taken in groups of `group`, and a group's units heaviest query
// tile first: the CTAs running at one time then read the K/V of about one group, which stays in L2.
OMNI_DEV void unit_of(int batch, int heads, int qtiles, int group, int u, int& b, int& h, int& qt) {
  const int bh_count = batch * heads;
  const int per_group = group * qtiles;
  const int g0 = (u / per_group) * group;
  const int gsize = min(group, bh_count - g0);
  const int r = u - g0 * qtiles;
  qt = qtiles - 1 - r / gsize;
  const int bh = g0 + r % gsize;
  b = bh / heads;
  h = bh % heads;
}

// A precomputed assignment of units to CTAs (kernel parameters): CTA c runs unit[start[c]] .. unit[start[c+1] - 1]
// in that order. The host builds it by list scheduling in the order unit_of numbers the units (each unit goes to
// the CTA that is free first, by a cost of its key tiles plus a unit's fixed cost), which keeps the CTAs' end times
// within about 1% where a round-robin assignment spreads them by 7-8% (config 4); the units a CTA runs at one time
// still belong to about one group. Shapes with more units than it holds, or grids larger than it covers, run
// round-robin (u = c, c + grid, ...).
constexpr int kSchedUnits = 4096;
constexpr int kSchedCtas = 160;
struct Sched {
  int on;
  uint16_t start[kSchedCtas + 1];
  uint16_t unit[kSchedUnits];
};

// The CTA's n-th unit, or -1 past its last.
OMNI_DEV int cta_unit(const Sched& s, int units, int n) {
  if (!s.on) {
    const int u = (int)blockIdx.x + n * (int)gridDim.x;
    return u < units ? u : -1;
  }
  const int k = (int)s.start[blockIdx.x] + n;
  return k < (int)s.start[blockIdx.x + 1] ? (int)s.unit[k] : -1;
}

}  // namespace pfx

// (row, head) pairs per scheduling group of the prefill kernels (prefill.cu).
int prefill_group(int bh_count);

// The list schedule of a prefill's units over `grid` CTAs (cached per shape; prefill.cu), or nullptr where the
// shape is past what a schedule holds: then the kernels run round-robin (prefill_round_robin()).
const pfx::Sched* prefill_schedule(int batch, int heads, int qtiles, int group, int grid);
const pfx::Sched& prefill_round_robin();

}  // namespace omni
