// Device helpers shared by the paged-MHA kernels: mbarriers with bounded waits, TMA tensor
// loads, tcgen05 (TMEM + UMMA) wrappers, FP16/BF16 unpacking and exp2.
//
// Every wait on an mbarrier is bounded by a global-timer budget carried in the launch
// parameters; on expiry the waiting thread records FGW_ERR_DEVICE_TIMEOUT in the workspace
// error word and the kernel unwinds instead of spinning forever.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "fgw_mha.h"

namespace fgw {

constexpr float kLog2e = 1.4426950408889634f;
// Split-KV partial LSE sentinel: a partition that saw no key publishes this value
// (the reference's -1e30, kept in the log2 domain used here); anything at or below
// kValidLse carries zero weight in the merge.
constexpr float kEmptyLse = -1.0e30f;
constexpr float kValidLse = -1.0e29f;

// Workspace header (first 256 bytes of every workspace).
struct WorkspaceHeader {
  int32_t error;        // first fgw_status recorded by a device thread, 0 when clean
  int32_t error_site;   // which wait gave up (kernel-defined id)
  uint32_t finished;    // decode kernel's dynamic deal: CTAs that have drawn their last item
  uint32_t pad0;
  unsigned long long next_item;  // decode kernel's dynamic deal: next whole item to hand out
  uint32_t pad[58];
};
static_assert(sizeof(WorkspaceHeader) == 256, "workspace header is 256 bytes");

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_error(WorkspaceHeader* ws, int code, int site) {
  if (ws != nullptr && atomicCAS(&ws->error, 0, code) == 0) {
    ws->error_site = site;
  }
}

// ---------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for the phase with the given parity to complete. Returns false if the budget ran
// out first (the caller records the error and unwinds).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t budget_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i) {
      if (mbar_try_wait(bar, parity)) return true;
    }
    if (global_timer_ns() - start > budget_ns) return false;
  }
}

// One request's block-table row as seen by a converged warp: the entries of a 32-page window, one per lane, read
// ahead of use and broadcast per lookup, so a producer's table reads leave its per-box path. Every lane must call
// both members with the same arguments; page() re-reads the window only when the page leaves it.
struct TableWindow {
  const int32_t* row;
  int width, base, entry;
  __device__ __forceinline__ void init(const int32_t* row_, int width_, int first_page, int lane) {
    row = row_;
    width = width_;
    base = first_page & ~31;
    entry = (base + lane < width) ? row[base + lane] : 0;
  }
  __device__ __forceinline__ int page(int pg, int lane) {
    if ((pg & ~31) != base) {
      base = pg & ~31;
      entry = (base + lane < width) ? row[base + lane] : 0;
    }
    return __shfl_sync(0xffffffffu, entry, pg & 31);
  }
};

// Named barrier over a subset of warps (id 0 is __syncthreads). These are the aligned forms: every lane of a
// warp executes them together, so callers reconverge the warp (__syncwarp) first.
__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Arrival on a named barrier without waiting (the waiting side calls named_barrier_sync with the same count).
__device__ __forceinline__ void named_barrier_arrive(uint32_t id, uint32_t threads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------------------------------
// TMA (tiled tensor loads, no cluster broadcast)
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_hint(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                                 int z, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, "
      "%4, %5}], [%2], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// ---------------------------------------------------------------------------------------
// Element conversions
// ---------------------------------------------------------------------------------------
template <typename T>
struct ElemTraits;

template <>
struct ElemTraits<__nv_bfloat16> {
  static constexpr int kUmmaFormat = 1;  // BF16 in the UMMA instruction descriptor
  __device__ __forceinline__ static float2 unpack2(uint32_t bits) {
    return make_float2(__uint_as_float(bits << 16), __uint_as_float(bits & 0xffff0000u));
  }
  __device__ __forceinline__ static uint32_t pack2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __device__ __forceinline__ static __nv_bfloat16 from_float(float x) { return __float2bfloat16_rn(x); }
  // acc + the two packed values, each added in FP32 (sm_100 mixed-precision add)
  __device__ __forceinline__ static float2 add2(float2 acc, uint32_t bits) {
    asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\tadd.rn.f32.bf16 %0, lo, %0;\n\t"
        "add.rn.f32.bf16 %1, hi, %1;\n\t}" : "+f"(acc.x), "+f"(acc.y) : "r"(bits));
    return acc;
  }
};

template <>
struct ElemTraits<__half> {
  static constexpr int kUmmaFormat = 0;  // F16
  __device__ __forceinline__ static float2 unpack2(uint32_t bits) {
    __half2 h = *reinterpret_cast<__half2*>(&bits);
    return __half22float2(h);
  }
  __device__ __forceinline__ static uint32_t pack2(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __device__ __forceinline__ static __half from_float(float x) { return __float2half_rn(x); }
  __device__ __forceinline__ static float2 add2(float2 acc, uint32_t bits) {
    asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\tadd.rn.f32.f16 %0, lo, %0;\n\t"
        "add.rn.f32.f16 %1, hi, %1;\n\t}" : "+f"(acc.x), "+f"(acc.y) : "r"(bits));
    return acc;
  }
};

// 2^x through the SFU's approximate base-2 exponential (ex2.approx, flush-to-zero):
// ex2(-inf) = +0, which the online softmax relies on for masked scores.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for a pair on the FMA pipe instead of the SFU, for x in [-127, 2^22): Cody-Waite style range
// reduction x = n + f with n = round(x), f in [-0.5, 0.5] (rounding by adding 1.5 * 2^23), then a
// degree-3 polynomial for 2^f, and 2^n applied by adding n to the exponent field. Inputs below -127 are
// clamped (result ~6e-39). The coefficients are the minimax fit of the relative error on [-0.5, 0.5] that
// fit_exp2_poly.py (beside this header) computes by Lawson's iteratively reweighted least squares; max
// relative error 7.5e-5, below half an FP16 ulp.
__device__ __forceinline__ float2 poly_exp2_pair(float2 x) {
  const float2 magic = make_float2(12582912.0f, 12582912.0f);
  x.x = fmaxf(x.x, -127.0f);
  x.y = fmaxf(x.y, -127.0f);
  const float2 t = __fadd2_rn(x, magic);                                  // n in the low mantissa bits
  const float2 n = __fadd2_rn(t, make_float2(-12582912.0f, -12582912.0f));
  const float2 f = __fadd2_rn(x, make_float2(-n.x, -n.y));
  float2 p = make_float2(0.0551713221f, 0.0551713221f);
  p = __ffma2_rn(p, f, make_float2(0.242610544f, 0.242610544f));
  p = __ffma2_rn(p, f, make_float2(0.693260968f, 0.693260968f));
  p = __ffma2_rn(p, f, make_float2(0.999928117f, 0.999928117f));
  // (bits(t) << 23) == (n << 23) mod 2^32, since bits(t) = 0x4B400000 + n.
  const int bx = __float_as_int(p.x) + (__float_as_int(t.x) << 23);
  const int by = __float_as_int(p.y) + (__float_as_int(t.y) << 23);
  return make_float2(__int_as_float(bx), __int_as_float(by));
}

// Per-warpgroup register budgets (setmaxnreg); N is a multiple of 8 in [24, 256].
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ float fast_log2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// LSE-weighted merge of split-KV partials (the reference's merge, v7.py:317-371: running max, rescale,
// invalid splits weighted 0, denominator clamped at 1e-30), in three steps with every rounding spelled
// out, so merge_kernel and the decode kernel's fused merge produce the same bits.
// Split s of a row: updates the running max and weight total, returns the old accumulators' and the new
// partial's weights.
__device__ __forceinline__ void merge_split_weights(float lse, float& peak, float& total, float& w_old,
                                                    float& w_new) {
  const float next = fmaxf(peak, lse);
  w_old = fast_exp2(peak - next);
  w_new = lse > kValidLse ? fast_exp2(lse - next) : 0.f;
  total = __fmaf_rn(total, w_old, w_new);
  peak = next;
}
// One element's accumulator after split s (the partial value counts only when it carries weight). Callers
// load a chunk of splits' LSEs and partial values with independent loads first, then apply the steps in
// split order, so the loads overlap instead of forming a chain through the weights.
__device__ __forceinline__ float merge_split_accumulate(float acc, float w_old, float w_new, float partial) {
  return __fmaf_rn(acc, w_old, w_new != 0.f ? __fmul_rn(partial, w_new) : 0.f);
}
__device__ __forceinline__ float merge_split_finish(float acc, float total) {
  return __fmul_rn(acc, __fdiv_rn(1.f, fmaxf(total, 1e-30f)));
}

// ---------------------------------------------------------------------------------------
// Contiguous schedule: T units cut into G programs; program p owns units [start(p), start(p + 1)),
// start(p) = p (T / G) + min(p, T % G) (the reference's balanced plan, static_schedule.py:64-66). An item cut
// between programs q_first .. q_first + pieces - 1 leaves one partial per piece in two slots per program:
// slot 2 q for the piece a program starts with, 2 q + 1 for the one it ends with.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ long long program_start(long long total, int programs, int p) {
  return static_cast<long long>(p) * (total / programs) + min(static_cast<long long>(p), total % programs);
}

__device__ __forceinline__ int program_of(long long total, int programs, long long u) {
  const long long b = total / programs, r = total % programs;
  if (u < r * (b + 1)) return static_cast<int>(u / (b + 1));
  return static_cast<int>(r + (u - r * (b + 1)) / b);
}

// Whole work items dealt to the persistent CTAs in snake order: round r gives CTA c item r * ctas + c when r is
// even and r * ctas + ctas - 1 - c when r is odd. With the items in longest-request-first order this keeps every
// CTA's total close to the mean even with a few items per CTA (dealt round-robin, the CTAs that draw the first,
// longest item of every round become stragglers: 1.26x the mean against 1.07x snake-wise on the decode
// workload's lengths with four heads per GPU), and consecutive items (the heads of one request) still run at the
// same time on neighbouring CTAs, which read the same tokens' rows together.
__device__ __forceinline__ long long snake_item(long long round) {
  return round * gridDim.x + ((round & 1) ? gridDim.x - 1 - blockIdx.x : blockIdx.x);
}

// Slot of piece k of an item whose first piece is held by program q_first; first_extra = 1 when the item
// starts inside q_first's range (that piece is q_first's last piece), 0 when it starts at the range's start.
__device__ __forceinline__ long long piece_slot(int q_first, int first_extra, int k) {
  return 2ll * q_first + first_extra + (k == 0 ? 0 : 2 * k - first_extra);
}

// ---------------------------------------------------------------------------------------
// tcgen05: TMEM allocation, UMMA issue/commit, TMEM loads and stores
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

// Programmatic dependent launch: a kernel launched with launch_after_plan may start its set-up while the plan
// kernel before it on the stream still runs; it reads what the plan wrote only after grid_dependency_wait(), which
// returns once that kernel has completed and its writes are visible. The plan lets its dependent start at once.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dependents_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

__device__ __forceinline__ void tc_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T (K-major B) for kind::f16, one CTA.
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// UMMA issue with each shared-memory descriptor passed as its two 32-bit words (see umma_desc_lo /
// umma_desc_hi), so an issue loop only adds an offset to the low word per instruction. umma_f16_ss_w reads A
// from shared memory; umma_f16_ts_w reads A (M x K, K-major) from tensor memory, one row per lane, two 16-bit
// elements per 32-bit column (element 2c in the low half of column c).
__device__ __forceinline__ void umma_f16_ss_w(uint32_t d_tmem, uint32_t a_lo, uint32_t a_hi, uint32_t b_lo,
                                              uint32_t b_hi, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\t"
      "mov.b64 da, {%1, %2};\n\t"
      "mov.b64 db, {%3, %4};\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %5, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_f16_ts_w(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t b_hi,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 db;\n\t"
      "mov.b64 db, {%2, %3};\n\t"
      "setp.ne.b32 p, %5, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %4, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on the mbarrier when every UMMA issued so far by this thread has completed.
// One lane of a converged warp (elect.sync): the issuing lane for the warp-wide tcgen05 issue helpers below.
__device__ __forceinline__ uint32_t elect_one_sync() {
  uint32_t pred = 0;
  asm volatile("{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}\n" : "=r"(pred));
  return pred;
}
// tcgen05.mma / commit executed by a whole converged warp and issued by the elected lane only, so the operands
// can stay warp-uniform.
__device__ __forceinline__ void umma_f16_ss_e(uint32_t leader, uint32_t d_tmem, uint32_t a_lo, uint32_t a_hi,
                                              uint32_t b_lo, uint32_t b_hi, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b64 da, db;\n\t"
      "setp.ne.b32 e, %7, 0;\n\t"
      "mov.b64 da, {%1, %2};\n\t"
      "mov.b64 db, {%3, %4};\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %5, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate), "r"(leader)
      : "memory");
}
__device__ __forceinline__ void umma_f16_ts_e(uint32_t leader, uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo,
                                              uint32_t b_hi, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b64 db;\n\t"
      "setp.ne.b32 e, %6, 0;\n\t"
      "mov.b64 db, {%2, %3};\n\t"
      "setp.ne.b32 p, %5, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %4, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate), "r"(leader)
      : "memory");
}
__device__ __forceinline__ void umma_commit_e(uint32_t leader, uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\tsetp.ne.b32 e, %1, 0;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(smem_u32(bar)),
      "r"(leader)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives row (lane_base + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 64 consecutive 32-bit columns (one instruction for half a 128-column score row).
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, "
      "%36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, "
      "%57, %58, %59, %60, %61, %62, %63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]),
        "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]),
        "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]),
        "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]),
        "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st4(uint32_t taddr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(r0), "r"(r1),
               "r"(r2), "r"(r3)
               : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Shared-memory matrix descriptor for tcgen05.mma (SM100 format, version 1).
//   start: byte address in shared memory; lbo/sbo: byte offsets; swizzle: 0 none, 2 = 128B.
__device__ __forceinline__ uint64_t umma_smem_desc(uint32_t start, uint32_t lbo, uint32_t sbo, uint32_t swizzle) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((start >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for SM100
  d |= static_cast<uint64_t>(swizzle & 0x7u) << 61;
  return d;
}

// The two 32-bit words of umma_smem_desc. Low word: start address >> 4 (bits 0-13) and leading byte
// offset >> 4 (bits 16-29). High word: stride byte offset >> 4 (bits 0-13), descriptor version 1 (bit 14)
// and the swizzle mode (bits 29-31). Adding (byte offset >> 4) to the low word moves the start address;
// shared-memory addresses stay below 2^18, so the sum never carries into the leading-offset field.
__device__ __forceinline__ uint32_t umma_desc_lo(uint32_t start, uint32_t lbo) {
  return ((start >> 4) & 0x3FFFu) | (((lbo >> 4) & 0x3FFFu) << 16);
}

__host__ __device__ constexpr uint32_t umma_desc_hi(uint32_t sbo, uint32_t swizzle) {
  return ((sbo >> 4) & 0x3FFFu) | (1u << 14) | ((swizzle & 0x7u) << 29);
}

// Instruction descriptor for kind::f16 with FP32 accumulation.
//   fmt: 0 = F16, 1 = BF16 (same for A and B); a_mn/b_mn: 1 when the operand is MN-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int fmt, int m, int n, int a_mn, int b_mn) {
  return (1u << 4)                                  // D format F32
         | (static_cast<uint32_t>(fmt) << 7)        // A format
         | (static_cast<uint32_t>(fmt) << 10)       // B format
         | (static_cast<uint32_t>(a_mn) << 15)      // A major
         | (static_cast<uint32_t>(b_mn) << 16)      // B major
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

}  // namespace fgw
