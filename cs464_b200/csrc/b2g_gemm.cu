// b2g_gemm.cu — the sm_100a GEMM family C[M,N] = A[M,K] · B[K,N] (fp16/bf16 in, fp32 accumulate) and its C ABI.
//
// One persistent, warp-specialised kernel covers the whole config space; tile shape, K step, ring depth, L2 grouping,
// split-K and operand layout are runtime parameters, so no config needs a compile of its own (the reference compiles
// one Triton kernel per config, kernels/triton_matmul.py:38-82). Per CTA:
//   warp 0        TMA producer: loads A/B tiles (128-byte swizzle) into a `stages`-deep shared-memory ring
//   warp 1        TMEM owner + MMA issuer: tcgen05.mma kind::f16, fp32 accumulators in tensor memory,
//                 double-buffered when two accumulators fit the 512 TMEM columns
//   warps 2..     epilogue: tcgen05.ld -> convert -> global store (fp16/bf16 C, or fp32 split-K partials)
// The tile order follows the reference's grouped-M L2 swizzle (kernels/triton_matmul.py:50-56). SPLIT_K > 1 writes
// fp32 partials to a [SPLIT_K, M, N] workspace that a second kernel sums in fixed order, so results are bitwise
// reproducible as in the reference (kernels/triton_matmul.py:6-7, :85-92).
//
// Skinny M (BLOCK_M <= 64) swaps the operands: the tensor core's 128-row side runs over N (B^T as the "A" operand,
// read N-major) and its narrow N side over M, so a 16-row activation still drives full-width MMAs.
//
// Every wait on an mbarrier is bounded (%globaltimer); on expiry the kernel records a code in the caller's status
// word, tells the other roles to stop, drains its own in-flight copies and MMAs, frees tensor memory and returns.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "b2g.h"
#include "b2g_ptx.cuh"

#ifndef B2G_SOURCE_HASH
#define B2G_SOURCE_HASH "unknown"
#endif
#define B2G_VERSION_STR "b2g-sm100a-0.1"

namespace b2g {

constexpr int kMaxStages = 16;
constexpr uint32_t kCtlBytes = 1024;   // control block (barriers, flags) at the start of dynamic shared memory
constexpr uint32_t kAlignSlack = 1024;  // data ring starts on the next 1024-byte boundary
constexpr uint64_t kWaitTimeoutNs = 1000000000ull;  // 1 s per wait: far above any legal stall
constexpr uint64_t kDrainTimeoutNs = 50000000ull;   // 50 ms to drain in-flight work after an abort
constexpr size_t kMaxSmemPerCta = 232448;          // sm_100 opt-in maximum dynamic shared memory per block
constexpr int kDefaultSmCount = 148;                // B200, when no device is current (host-only sizing)
constexpr int kMaxRedCluster = 8;                   // split-K summed in a cluster of at most 8 CTAs (portable size)
constexpr int64_t kMaxRedElems = 8192;              // ... for tiles of at most 8192 fp32 partials (32 KB) per CTA

// control block layout (byte offsets)
constexpr uint32_t OFF_FULL = 0;      // kMaxStages x u64
constexpr uint32_t OFF_EMPTY = 128;   // kMaxStages x u64
constexpr uint32_t OFF_TFULL = 256;   // 2 x u64: accumulator ready for the epilogue
constexpr uint32_t OFF_TEMPTY = 272;  // 2 x u64: accumulator drained by the epilogue
constexpr uint32_t OFF_DRAIN = 288;   // u64: all MMAs of this CTA complete
constexpr uint32_t OFF_TMEM = 296;    // u32: tensor-memory base address written by tcgen05.alloc
constexpr uint32_t OFF_ABORT = 300;   // u32: set when any role gave up waiting
constexpr uint32_t OFF_EPISYNC = 304; // u64: epilogue-warps rendezvous (stream-K fix-up), bounded like every wait

// status codes written to the caller's device status word
constexpr int kStatusProducerTimeout = 0x101;
constexpr int kStatusMmaTimeout = 0x102;
constexpr int kStatusEpilogueTimeout = 0x103;
constexpr int kStatusStreamkTimeout = 0x104;

enum OutKind : int32_t { OUT_F16 = 0, OUT_BF16 = 1, OUT_F32_PARTIAL = 2 };

// n / d for 0 <= n < 2^31 by a multiply-high and a shift (round-up reciprocal, Granlund & Montgomery 1994): the
// tile decode runs on one thread per role, where a chain of hardware-less 32-bit divisions costs hundreds of cycles.
struct FastDiv {
  uint32_t d, m, s;
};

inline FastDiv make_fastdiv(uint32_t d) {
  FastDiv f;
  f.d = d < 1 ? 1 : d;
  f.s = 0;
  while ((uint64_t(1) << f.s) < f.d) ++f.s;
  f.m = static_cast<uint32_t>(((uint64_t(1) << 32) * ((uint64_t(1) << f.s) - f.d)) / f.d + 1);
  return f;
}

__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) {
  return static_cast<uint32_t>((static_cast<uint64_t>(__umulhi(n, f.m)) + n) >> f.s);
}

// Kernel parameters, in the MMA's orientation: D[i, j] with i over `rows_a` (tensor-memory lanes) and j over
// `rows_b` (tensor-memory columns). Without the swap i = m, j = n; with it i = n, j = m.
struct KParams {
  int32_t rows_a, rows_b, K;
  int32_t tile_m, tile_n, bk, stages;
  int32_t cta_m, cta_n;  // A and B rows one CTA loads (tile_m, tile_n; halves of them in a CTA pair)
  int32_t group_m, split_k;
  int32_t tiles_m, tiles_n, num_kb, units;
  // divisors of the tile decode: split_k, group_m * tiles_n, group_m, and the last group's height
  FastDiv fd_split, fd_group, fd_gm, fd_last;
  int32_t last_group_first;  // first tile row of the last (possibly shorter) group
  int32_t a_mn_major, b_mn_major;
  int32_t a_3d, b_3d;  // MN-major operand read by one 3-D copy per K block (all its 64-wide column groups)
  uint32_t idesc;
  uint32_t a_stage_bytes, b_stage_bytes;
  uint32_t acc_cols, num_acc, tmem_cols;
  void* out;
  int64_t out_si, out_sj, out_split_stride;
  int32_t out_kind, vec_ok;
  // Row-major output written through a 4 KB shared staging tile per epilogue warp (non-swapped tiles, 16-byte rows,
  // whole 16-byte pieces): the staging area starts `epi_stage_off` bytes after the operand ring.
  int32_t stage_c;
  uint32_t epi_stage_off;
  int* status;
  uint64_t timeout_ns;
  // stream-K: workers (CTAs, or CTA pairs) share sk_iters = tiles * num_kb K blocks in equal contiguous slices; a tile
  // split over several workers is finished by the worker holding its first K block (its owner), which adds the other
  // workers' fp32 partials (one slot of cta_m x tile_n per CTA) in K order after their flags are raised.
  int32_t streamk;
  int32_t sk_dp_tiles;  // tiles 0 .. sk_dp_tiles-1 run whole, data-parallel (full waves)
  int32_t sk_workers;   // workers 0 .. sk_workers-1 share the remaining tiles' K blocks
  int64_t sk_iters;     // (tiles - sk_dp_tiles) * num_kb
  float* sk_slots;
  int* sk_flags;
  // split-K summed inside a cluster of the SPLIT_K CTAs of a tile (lean form only): each CTA leaves its fp32 partial
  // in its own shared memory (laid out along C's contiguous direction: [j][i] when red_imajor, else [i][j], rows
  // padded by 4 floats), then CTA r sums slice r of the tile over every CTA's partial in split order and writes C.
  int32_t red_cluster, red_imajor;
};

struct Unit {
  int tm, tn, split, kb0, kb1;
  int tile;  // tile index in the grouped order (stream-K)
};

// (tm, tn) of the t-th tile in the grouped-M L2 order (kernels/triton_matmul.py:50-56)
__device__ __forceinline__ void tile_coords(const KParams& p, int t, int& tm, int& tn) {
  const uint32_t gid = fdiv(static_cast<uint32_t>(t), p.fd_group);
  const int first = static_cast<int>(gid) * p.group_m;
  const int r = t - static_cast<int>(gid) * p.group_m * p.tiles_n;
  const FastDiv& g = first == p.last_group_first ? p.fd_last : p.fd_gm;
  const int q = static_cast<int>(fdiv(static_cast<uint32_t>(r), g));
  tm = first + (r - q * static_cast<int>(g.d));
  tn = q;
}

__device__ __forceinline__ Unit decode_unit(const KParams& p, int u) {
  Unit w;
  if (p.split_k == 1) {
    w.split = 0;
    w.tile = u;
    w.kb0 = 0;
    w.kb1 = p.num_kb;
  } else {
    const int t = static_cast<int>(fdiv(static_cast<uint32_t>(u), p.fd_split));
    w.split = u - t * p.split_k;
    w.tile = t;
    // split * num_kb / split_k: below 2^31 because split_k * num_kb is (checked when the plan is made)
    const uint32_t nkb = static_cast<uint32_t>(p.num_kb);
    w.kb0 = static_cast<int>(fdiv(static_cast<uint32_t>(w.split) * nkb, p.fd_split));
    w.kb1 = static_cast<int>(fdiv(static_cast<uint32_t>(w.split + 1) * nkb, p.fd_split));
  }
  tile_coords(p, w.tile, w.tm, w.tn);
  return w;
}

// First K-block iteration (global: tile * num_kb + kb) of stream-K worker `w`'s shared slice.
__device__ __forceinline__ int64_t sk_start(const KParams& p, int64_t w) {
  return static_cast<int64_t>(p.sk_dp_tiles) * p.num_kb + w * p.sk_iters / p.sk_workers;
}

// The sequence of work items of one worker: units worker, worker + workers, ... (tiles or split-K units). With
// stream-K: first the (tile, K range) segments of its slice of the shared K blocks, then its whole tiles of the
// data-parallel waves. Shared segments first: an owner's fix-up (waiting for its contributors' partials, adding them)
// then runs in its epilogue while its MMA warp already works on the next tile, instead of after the last one; and a
// contributor never waits, so the owners' waits all end. Every role walks the same sequence.
struct Cursor {
  int64_t it, hi;
  int u;
};

__device__ __forceinline__ void cursor_init(const KParams& p, Cursor& c, int worker, int workers) {
  (void)workers;
  c.u = worker;
  if (p.streamk) {
    const bool shares = worker < p.sk_workers;
    c.it = shares ? sk_start(p, worker) : 0;
    c.hi = shares ? sk_start(p, worker + 1) : 0;
  }
}

__device__ __forceinline__ bool cursor_next(const KParams& p, Cursor& c, int workers, Unit& w) {
  if (p.streamk) {
    if (c.it < c.hi) {  // a (tile, K range) segment of this worker's slice of the shared K blocks
      const int64_t t = c.it / p.num_kb;
      w.kb0 = static_cast<int>(c.it - t * p.num_kb);
      w.kb1 = static_cast<int>(min(static_cast<int64_t>(p.num_kb), w.kb0 + (c.hi - c.it)));
      w.tile = static_cast<int>(t);
      w.split = 0;
      tile_coords(p, w.tile, w.tm, w.tn);
      c.it += w.kb1 - w.kb0;
      return true;
    }
    if (c.u < p.sk_dp_tiles) {  // a whole tile of the data-parallel waves
      w.tile = c.u;
      w.split = 0;
      w.kb0 = 0;
      w.kb1 = p.num_kb;
      tile_coords(p, w.tile, w.tm, w.tn);
      c.u += workers;
      return true;
    }
    return false;
  }
  if (c.u >= p.units) return false;
  w = decode_unit(p, c.u);
  c.u += workers;
  return true;
}

// Bounded wait: true once the phase with `parity` completed; false if another role aborted or `timeout_ns` passed
// (then this role sets the abort flag and records `code`).
// The slow path suspends on the barrier in slices of at most a quarter of the limit (at most 1 ms), so the limit
// holds to within a slice whatever the hardware's own suspend time is.
__device__ __noinline__ bool wait_phase(uint32_t bar, uint32_t parity, volatile uint32_t* abort_flag, int* status,
                                        uint64_t timeout_ns, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint32_t slice = static_cast<uint32_t>(timeout_ns / 4 < 1000000ull ? timeout_ns / 4 : 1000000ull);
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    if (mbar_try_wait_hint(bar, parity, slice)) return true;
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 > timeout_ns) {
      *abort_flag = 1u;
      if (status) atomicCAS(status, 0, code);
      return false;
    }
  }
}

// Wait for a phase during teardown, ignoring the abort flag, for at most `limit_ns`.
__device__ __noinline__ void drain_phase(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > limit_ns) return;
  }
}

// ---- stream-K fix-up flags (global memory, one int per CTA slot)
__device__ __forceinline__ int flag_acquire(const int* f) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  return v;
}

__device__ __forceinline__ void flag_release(int* f, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}

// Bounded wait for a contributor's flag; false (and the stream-K status code) after timeout_ns.
__device__ __noinline__ bool flag_wait(const int* f, volatile uint32_t* abort_flag, int* status, uint64_t timeout_ns) {
  if (flag_acquire(f) == 1) return true;
  const uint64_t t0 = global_timer_ns();
  while (flag_acquire(f) != 1) {
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 > timeout_ns) {
      *abort_flag = 1u;
      if (status) atomicCAS(status, 0, kStatusStreamkTimeout);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ uint32_t cvt_pair(float a, float b, int bf16) {
  if (bf16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint16_t cvt_one(float a, int bf16) {
  if (bf16) {
    __nv_bfloat16 h = __float2bfloat16_rn(a);
    return *reinterpret_cast<uint16_t*>(&h);
  }
  __half h = __float2half_rn(a);
  return *reinterpret_cast<uint16_t*>(&h);
}

// Store `ncol` (16 or 32) accumulator values of row i = `row`, columns j = col0.. of D.
__device__ __forceinline__ void store_chunk(const KParams& p, int split, int64_t row, int64_t col0, int ncol,
                                            const uint32_t (&v)[32]) {
  if (row >= p.rows_a) return;
  const bool full = p.vec_ok && (col0 + ncol <= p.rows_b);
  if (p.out_kind == OUT_F32_PARTIAL) {
    float* o = static_cast<float*>(p.out) + static_cast<int64_t>(split) * p.out_split_stride + row * p.out_si;
    if (full) {
      float4* dst = reinterpret_cast<float4*>(o + col0);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (q * 4 < ncol)
          dst[q] = make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                               __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (j < ncol && col0 + j < p.rows_b) o[(col0 + j) * p.out_sj] = __uint_as_float(v[j]);
      }
    }
    return;
  }
  const int bf = p.out_kind == OUT_BF16;
  uint16_t* o = static_cast<uint16_t*>(p.out) + row * p.out_si;
  if (full) {
    uint4* dst = reinterpret_cast<uint4*>(o + col0);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (q * 8 < ncol) {
        uint4 w;
        w.x = cvt_pair(__uint_as_float(v[8 * q + 0]), __uint_as_float(v[8 * q + 1]), bf);
        w.y = cvt_pair(__uint_as_float(v[8 * q + 2]), __uint_as_float(v[8 * q + 3]), bf);
        w.z = cvt_pair(__uint_as_float(v[8 * q + 4]), __uint_as_float(v[8 * q + 5]), bf);
        w.w = cvt_pair(__uint_as_float(v[8 * q + 6]), __uint_as_float(v[8 * q + 7]), bf);
        dst[q] = w;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j < ncol && col0 + j < p.rows_b) o[(col0 + j) * p.out_sj] = cvt_one(__uint_as_float(v[j]), bf);
    }
  }
}

// 32 rows x 128 bytes of output through shared memory: lane r writes row r's eight 16-byte pieces (four at a time,
// from `j0`), with the piece index XOR-ed by (row & 7), which keeps both the row-wise writes and the piece-wise reads
// free of bank conflicts; `stage_flush` then writes four whole 128-byte row segments per global store instruction
// instead of 32 scattered 16-byte pieces (the load/store unit, not HBM, bounds the direct path). `rows` / `pieces`:
// how many of the 32 rows and 8 pieces lie inside C.
__device__ __forceinline__ void stage_write4(uint32_t stg, int lane, int j0, const uint4 (&pc)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) st_shared_v4(stg + lane * 128 + (((j0 + j) ^ (lane & 7)) << 4), pc[j]);
}

__device__ __forceinline__ void stage_flush(uint32_t stg, int lane, uint8_t* base, int64_t row_bytes, int rows,
                                            int pieces) {
  __syncwarp();
  const int pp = lane & 7;
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    const int rr = 4 * s + (lane >> 3);
    const uint4 x = ld_shared_v4(stg + rr * 128 + ((pp ^ (rr & 7)) << 4));
    if (rr < rows && pp < pieces) *reinterpret_cast<uint4*>(base + rr * row_bytes + pp * 16) = x;
  }
  __syncwarp();
}

// One CTA (PAIR = 0) or one CTA of a pair (PAIR = 1, cluster of 2, cta_group::2 MMAs of M = 256).
// LEAN = 1 (single CTAs only): the launch has one CTA per work unit (no stream-K, split-K reduced by the separate
// kernel), so the unit walk, the stream-K fix-up and the in-kernel split-K sum are compiled out. A small GEMM's time is
// mostly fixed cost, and much of that is fetching the instructions its warps execute from a cold cache: the lean form
// executes far fewer of them.
template <int EPI_WARPS, int PAIR, int LEAN = 0>
__global__ void __launch_bounds__((2 + EPI_WARPS) * 32, 1)
    gemm_kernel(const __grid_constant__ KParams p, const __grid_constant__ CUtensorMap tma_a,
                const __grid_constant__ CUtensorMap tma_b) {
  static_assert(!(LEAN && PAIR), "the lean form is single-CTA only");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // Let a programmatically dependent launch (the split-K reduce, or the next GEMM) be scheduled once every CTA of this
  // grid is running; the dependent waits for this grid's completion before it touches global memory.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // This grid may itself be such a dependent: its set-up (barriers, tensor memory, descriptor prefetch) overlaps the
  // previous kernel's tail, and every thread waits for that kernel to complete (its writes visible) before its first
  // global access — A and B may be its outputs, and C or the workspace its inputs. Without the launch attribute the
  // wait returns at once.
  const uint32_t ctl = smem_addr(smem_raw);
  const uint32_t data = (ctl + kCtlBytes + 1023u) & ~1023u;
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem_raw + OFF_ABORT);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t stage_bytes = p.a_stage_bytes + p.b_stage_bytes;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int first_unit = PAIR ? static_cast<int>(cluster_id_x()) : static_cast<int>(blockIdx.x);
  const int unit_step = PAIR ? static_cast<int>(num_clusters_x()) : static_cast<int>(gridDim.x);
  // every role walks the same sequence of units; the lean form has exactly one, this CTA's
  auto next_unit = [&](Cursor& c, Unit& w) -> bool {
    if constexpr (LEAN) {
      if (c.u < 0) return false;
      w = decode_unit(p, c.u);
      c.u = -1;
      return true;
    } else {
      return cursor_next(p, c, unit_step, w);
    }
  };

  // ---------------------------------------------------------------- TMA producer state (thread 0)
  // The producer walks (unit, K block) pairs in order; `produce(n)` issues copies until n stages are in flight in
  // total or the work runs out, so its first stages can go out before the block-wide barrier below.
  Cursor pc;
  cursor_init(p, pc, first_unit, unit_step);
  int pkb = 0, pkb1 = 0, prow_a = 0, prow_b = 0;
  int ps = 0, pissued = 0;
  uint32_t pph = 0;
  bool pok = true;
  const uint32_t tx_bytes = PAIR ? 2u * stage_bytes : stage_bytes;
  auto produce = [&](int max_issue, uint32_t full_leader) {
    while (pok && pissued < max_issue) {
      while (pkb >= pkb1) {  // next unit with at least one K block
        Unit w;
        if (!next_unit(pc, w)) return;
        pkb = w.kb0;
        pkb1 = w.kb1;
        prow_a = w.tm * p.tile_m + static_cast<int>(rank) * p.cta_m;
        prow_b = w.tn * p.tile_n + static_cast<int>(rank) * p.cta_n;
      }
      const uint32_t empty = ctl + OFF_EMPTY + 8 * ps;
      if (!mbar_try_wait(empty, pph ^ 1u) &&
          !wait_phase(empty, pph ^ 1u, abort_flag, p.status, p.timeout_ns, kStatusProducerTimeout)) {
        pok = false;
        return;
      }
      const uint32_t full = ctl + OFF_FULL + 8 * ps;
      // the pair's leader counts both CTAs' bytes on its own barrier; the peer only issues copies
      if (leader) mbar_arrive_expect_tx(full, tx_bytes);
      const uint32_t full_c = full_leader + 8 * ps;
      const uint32_t sa = data + ps * stage_bytes;
      const uint32_t sb = sa + p.a_stage_bytes;
      const int k0 = pkb * p.bk;
      if (p.a_3d) {
        if (PAIR) tma_load_3d_pair(sa, &tma_a, full_c, 0, k0, prow_a / 64);
        else tma_load_3d(sa, &tma_a, full, 0, k0, prow_a / 64);
      } else if (p.a_mn_major) {
        for (int a = 0; a < p.cta_m / 64; ++a) {
          if (PAIR) tma_load_2d_pair(sa + a * p.bk * 128, &tma_a, full_c, prow_a + a * 64, k0);
          else tma_load_2d(sa + a * p.bk * 128, &tma_a, full, prow_a + a * 64, k0);
        }
      } else {
        for (int a = 0; a < p.bk / 64; ++a) {
          if (PAIR) tma_load_2d_pair(sa + a * p.cta_m * 128, &tma_a, full_c, k0 + a * 64, prow_a);
          else tma_load_2d(sa + a * p.cta_m * 128, &tma_a, full, k0 + a * 64, prow_a);
        }
      }
      if (p.b_3d) {
        if (PAIR) tma_load_3d_pair(sb, &tma_b, full_c, 0, k0, prow_b / 64);
        else tma_load_3d(sb, &tma_b, full, 0, k0, prow_b / 64);
      } else if (p.b_mn_major) {
        for (int a = 0; a < p.cta_n / 64; ++a) {
          if (PAIR) tma_load_2d_pair(sb + a * p.bk * 128, &tma_b, full_c, prow_b + a * 64, k0);
          else tma_load_2d(sb + a * p.bk * 128, &tma_b, full, prow_b + a * 64, k0);
        }
      } else {
        for (int a = 0; a < p.bk / 64; ++a) {
          if (PAIR) tma_load_2d_pair(sb + a * p.cta_n * 128, &tma_b, full_c, k0 + a * 64, prow_b);
          else tma_load_2d(sb + a * p.cta_n * 128, &tma_b, full, k0 + a * 64, prow_b);
        }
      }
      ++pissued;
      ++pkb;
      if (++ps == p.stages) {
        ps = 0;
        pph ^= 1u;
      }
    }
  };

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(ctl + OFF_FULL + 8 * s, 1);
      mbar_init(ctl + OFF_EMPTY + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(ctl + OFF_TFULL + 8 * b, 1);
      mbar_init(ctl + OFF_TEMPTY + 8 * b, (PAIR ? 2 : 1) * EPI_WARPS * 32);
    }
    mbar_init(ctl + OFF_DRAIN, 1);
    mbar_init(ctl + OFF_EPISYNC, EPI_WARPS * 32);
    *abort_flag = 0u;
    fence_mbar_init();
    // A single CTA issues its first stage while warp 1 allocates tensor memory: only this thread has touched the
    // barriers so far, and the other roles wait on them after the barrier below. One stage, not the whole ring:
    // issuing more delays the barrier, and with it the first MMA. A pair's copies signal the leader's barriers,
    // which exist only after the cluster barrier.
    if (!PAIR) {
      asm volatile("griddepcontrol.wait;" ::: "memory");
      produce(1, ctl + OFF_FULL);
    }
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(ctl + OFF_TMEM, p.tmem_cols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(ctl + OFF_TMEM, p.tmem_cols);
      tmem_relinquish();
    }
  }
  // Lane 0 of warp 0 may still be issuing its first copies: the warp converges first, because a block or cluster
  // barrier reached by part of a warp counts the whole warp as arrived.
  __syncwarp();
  tc_fence_before();
  if (PAIR) {
    cluster_sync();  // both CTAs' barriers initialised and tensor memory allocated before any cross-CTA signal
  } else {
    __syncthreads();
  }
  tc_fence_after();
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(smem_raw + OFF_TMEM);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (every CTA loads its own tiles)
    if (lane == 0) {
      produce(0x7fffffff, PAIR ? map_to_rank(ctl + OFF_FULL, 0) : ctl + OFF_FULL);
      if (!pok && leader) {
        // Let the copies already issued land before shared memory is released (the leader's barriers count the
        // pair's bytes).
        const int pending = min(pissued, p.stages);
        int ds = ps;
        uint32_t dph = pph;
        for (int i = 0; i < pending; ++i) {
          if (--ds < 0) {
            ds = p.stages - 1;
            dph ^= 1u;
          }
          drain_phase(ctl + OFF_FULL + 8 * ds, dph, kDrainTimeoutNs);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (the pair's leader issues for both)
    // The whole warp walks the loop and waits together; lane 0 alone issues the MMAs and commits (predicated), so
    // the warp stays converged and the descriptors uniform.
    if (leader) {
      int s = 0;
      uint32_t ph = 0;
      uint32_t acc = 0, acc_ph = 0;
      bool ok = true;
      // Descriptors of stage 0 / K step 0 / first 128 rows. Every other (stage, step, half) is a fixed byte offset
      // added, in 16-byte units, to the start-address field; shared addresses stay below 256 KB so the 14-bit field
      // never carries into the next one.
      const uint64_t adesc0 = sdesc_sw128(data, p.a_mn_major ? static_cast<uint32_t>(p.bk) * 128u : 16u, 1024u);
      const uint64_t bdesc0 =
          sdesc_sw128(data + p.a_stage_bytes, p.b_mn_major ? static_cast<uint32_t>(p.bk) * 128u : 16u, 1024u);
      const uint32_t stage16 = stage_bytes >> 4;
      // K step kk sits at (kk / 4) * step4 + (kk % 4) * step1: MN-major rows of 2048 B per 16 K, K-major 32 B per 16 K
      // inside a 64-wide swizzle atom and one atom (rows x 128 B) per 64 K.
      const uint32_t a_step4 = (p.a_mn_major ? 4u * 2048u : static_cast<uint32_t>(p.cta_m) * 128u) >> 4;
      const uint32_t a_step1 = (p.a_mn_major ? 2048u : 32u) >> 4;
      const uint32_t b_step4 = (p.b_mn_major ? 4u * 2048u : static_cast<uint32_t>(p.cta_n) * 128u) >> 4;
      const uint32_t b_step1 = (p.b_mn_major ? 2048u : 32u) >> 4;
      // second 128 rows of a 256-row single-CTA tile: two 64-row atoms on (MN-major) or 128 rows of 128 B (K-major)
      const uint32_t a_half16 = (p.a_mn_major ? 2u * static_cast<uint32_t>(p.bk) * 128u : 128u * 128u) >> 4;
      const bool two_halves = !PAIR && p.tile_m == 256;
      const int ksteps = p.bk / 16;
      // commits name each CTA's barrier by its shared::cluster address (the pair's leader signals both CTAs)
      const uint32_t empty0 = PAIR ? map_to_rank(ctl + OFF_EMPTY, 0) : ctl + OFF_EMPTY;
      const uint32_t empty1 = PAIR ? map_to_rank(ctl + OFF_EMPTY, 1) : 0u;
      const uint32_t tfull0 = PAIR ? map_to_rank(ctl + OFF_TFULL, 0) : ctl + OFF_TFULL;
      const uint32_t tfull1 = PAIR ? map_to_rank(ctl + OFF_TFULL, 1) : 0u;
      const uint32_t idesc = p.idesc;
      Cursor mc;
      cursor_init(p, mc, first_unit, unit_step);
      Unit w;
      while (ok && next_unit(mc, w)) {
        if (w.kb0 == w.kb1) continue;
        if (!mbar_try_wait(ctl + OFF_TEMPTY + 8 * acc, acc_ph ^ 1u) &&
            !wait_phase(ctl + OFF_TEMPTY + 8 * acc, acc_ph ^ 1u, abort_flag, p.status, p.timeout_ns,
                        kStatusMmaTimeout)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_base = tmem_base + acc * p.acc_cols;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          const uint32_t full = ctl + OFF_FULL + 8 * s;
          // TMA data is ordered by the barrier's byte count (both are async-proxy operations): no tcgen05 fence here
          if (!mbar_try_wait(full, ph) &&
              !wait_phase(full, ph, abort_flag, p.status, p.timeout_ns, kStatusMmaTimeout)) {
            ok = false;
            break;
          }
          const uint64_t a_s = adesc0 + s * stage16;
          const uint64_t b_s = bdesc0 + s * stage16;
          const uint32_t first = (kb == w.kb0) ? 0u : 1u;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            if (kk < ksteps) {
              const uint64_t ad = a_s + ((kk >> 2) * a_step4 + (kk & 3) * a_step1);
              const uint64_t bd = b_s + ((kk >> 2) * b_step4 + (kk & 3) * b_step1);
              const uint32_t accumulate = kk == 0 ? first : 1u;
              if (PAIR) {
                umma_f16_pair_w(d_base, ad, bd, idesc, accumulate);
              } else {
                umma_f16_w(d_base, ad, bd, idesc, accumulate);
                if (two_halves) umma_f16_w(d_base + p.tile_n, ad + a_half16, bd, idesc, accumulate);
              }
            }
          }
          if (PAIR) {
            umma_commit_pair_w(empty0 + 8 * s);
            umma_commit_pair_w(empty1 + 8 * s);
          } else {
            umma_commit_w(empty0 + 8 * s);
          }
          if (++s == p.stages) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        if (PAIR) {
          umma_commit_pair_w(tfull0 + 8 * acc);
          umma_commit_pair_w(tfull1 + 8 * acc);
        } else {
          umma_commit_w(tfull0 + 8 * acc);
        }
        if (++acc == p.num_acc) {
          acc = 0;
          acc_ph ^= 1u;
        }
      }
      // Every MMA this thread issued has finished before tensor memory is released.
      if (PAIR) umma_commit_pair_w(map_to_rank(ctl + OFF_DRAIN, 0));
      else umma_commit_w(ctl + OFF_DRAIN);
      drain_phase(ctl + OFF_DRAIN, 0, ok ? kWaitTimeoutNs : kDrainTimeoutNs);
    }
  } else {
    // ------------------------------------------------------------ epilogue (each CTA drains its own accumulator)
    const int e = warp - 2;
    const int q = warp & 3;  // tensor-memory lane quarter this warp may access
    const int grp = e >> 2;
    constexpr int kGroups = EPI_WARPS / 4;
    const int nchunks = (p.tile_n + 31) / 32;
    const int halves = PAIR ? 1 : p.tile_m / 128;
    const uint32_t tempty_leader = PAIR ? map_to_rank(ctl + OFF_TEMPTY, 0) : 0u;
    uint32_t acc = 0, acc_ph = 0;
    const int epi_tid = static_cast<int>(threadIdx.x) - 64;
    uint32_t sync_ph = 0;
    // rendezvous of the epilogue warps through an mbarrier: bounded, so a thread that gave up cannot strand the rest
    auto epilogue_sync = [&]() -> bool {
      mbar_arrive(ctl + OFF_EPISYNC);
      const bool ok = mbar_try_wait(ctl + OFF_EPISYNC, sync_ph) ||
                      wait_phase(ctl + OFF_EPISYNC, sync_ph, abort_flag, p.status, p.timeout_ns, kStatusEpilogueTimeout);
      sync_ph ^= 1u;
      return ok;
    };
    const int64_t slot_elems = static_cast<int64_t>(p.cta_m) * p.tile_n;
    // A stream-K slot holds a CTA's cta_m x tile_n fp32 partial as float4 pieces ordered [32-column chunk][piece of
    // 4 columns][row]: the 32 lanes of a warp (32 consecutive rows) store or load 512 contiguous bytes per
    // instruction. `piece0` = chunk * 8 + first piece, in pieces of cta_m float4s.
    auto slot_piece = [&](int64_t slot, int piece, int row_local) -> int64_t {
      return slot * (slot_elems / 4) + static_cast<int64_t>(piece) * p.cta_m + row_local;
    };
    // Stream-K owner: add the fp32 partials that contributors j0 .. j1-1 (later K blocks, in worker order) left for
    // `ncol` columns (32-column chunk `chunk`, row `row_local`) of their slots, in that fixed order.
    auto add_partials = [&](uint32_t (&v)[32], int chunk, int row_local, int ncol, int j0, int j1) {
      const float4* slots4 = reinterpret_cast<const float4*>(p.sk_slots);
      for (int j = j0; j < j1; ++j) {
        const int64_t slot = PAIR ? 2 * j + static_cast<int>(rank) : j;
        float4 x[8];  // the chunk's eight 16-byte pieces in flight together: one memory latency per contributor
#pragma unroll
        for (int k4 = 0; k4 < 8; ++k4)
          if (k4 * 4 < ncol) x[k4] = slots4[slot_piece(slot, chunk * 8 + k4, row_local)];
#pragma unroll
        for (int k4 = 0; k4 < 8; ++k4) {
          const int e = 4 * k4;
          if (e < ncol) {
            v[e] = __float_as_uint(__uint_as_float(v[e]) + x[k4].x);
            v[e + 1] = __float_as_uint(__uint_as_float(v[e + 1]) + x[k4].y);
            v[e + 2] = __float_as_uint(__uint_as_float(v[e + 2]) + x[k4].z);
            v[e + 3] = __float_as_uint(__uint_as_float(v[e + 3]) + x[k4].w);
          }
        }
      }
    };
    if (LEAN && p.red_cluster) {
      // This CTA's partial (its K range of the tile) into its shared memory: the operand ring is free once every MMA
      // has completed, which the accumulator barrier signals. The sum over the cluster follows the role branches.
      const Unit w = decode_unit(p, first_unit);
      const bool zero = w.kb0 == w.kb1;
      if (zero || wait_phase(ctl + OFF_TFULL, 0u, abort_flag, p.status, p.timeout_ns, kStatusEpilogueTimeout)) {
        if (!zero) tc_fence_after();
        for (int h = 0; h < halves; ++h) {
          const int i = h * 128 + q * 32 + lane;  // tile row (tensor-memory lane)
          for (int c = grp; c < nchunks; c += kGroups) {
            const int ncol = min(32, p.tile_n - c * 32);
            uint32_t v[32];
            if (zero) {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = 0u;
            } else {
              const uint32_t taddr = tmem_base + h * p.tile_n + c * 32 + (static_cast<uint32_t>(q * 32) << 16);
              if (ncol == 32) tmem_ld_32cols(taddr, v);
              else tmem_ld_16cols(taddr, v);
              tmem_ld_wait();
            }
            if (p.red_imajor) {  // [j][i]: the warp's 32 rows are 32 consecutive words of each column
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < ncol) st_shared_u32(data + ((c * 32 + j) * (p.tile_m + 4) + i) * 4u, v[j]);
            } else {  // [i][j]: rows 4 floats apart in banks, so each quarter-warp's 16-byte stores are conflict-free
#pragma unroll
              for (int k4 = 0; k4 < 8; ++k4)
                if (k4 * 4 < ncol)
                  st_shared_v4(data + (i * (p.tile_n + 4) + c * 32 + k4 * 4) * 4u,
                               make_uint4(v[4 * k4], v[4 * k4 + 1], v[4 * k4 + 2], v[4 * k4 + 3]));
            }
          }
        }
      }
    } else {
    Cursor ec;
    cursor_init(p, ec, first_unit, unit_step);
    Unit w;
    while (next_unit(ec, w)) {
      const bool zero = w.kb0 == w.kb1;
      // stream-K: a segment covering only part of its tile either contributes a partial (it does not hold the
      // tile's first K block) or owns the tile and adds the contributors' partials
      const bool partial = !LEAN && p.streamk && !(w.kb0 == 0 && w.kb1 == p.num_kb);
      const bool contrib = partial && w.kb0 > 0;
      const bool owner = partial && w.kb0 == 0;
      int j_end = first_unit + 1;  // contributors of an owned tile: workers first_unit + 1 .. j_end - 1
      if (!zero) {
        if (!wait_phase(ctl + OFF_TFULL + 8 * acc, acc_ph, abort_flag, p.status, p.timeout_ns,
                        kStatusEpilogueTimeout))
          break;
        tc_fence_after();
      }
      if (owner) {
        const int64_t tile_end = static_cast<int64_t>(w.tile + 1) * p.num_kb;
        while (j_end < p.sk_workers && sk_start(p, j_end) < tile_end) ++j_end;
        // one thread polls the contributors' flags; the bounded rendezvous then orders every thread after its
        // acquire loads
        if (epi_tid == 0) {
          for (int j = first_unit + 1; j < j_end; ++j) {
            if (sk_start(p, j) == sk_start(p, j + 1)) continue;  // empty slice: no partial
            if (!flag_wait(p.sk_flags + (PAIR ? 2 * j + static_cast<int>(rank) : j), abort_flag, p.status,
                           p.timeout_ns))
              break;
          }
        }
        epilogue_sync();
      }
      for (int h = 0; h < halves; ++h) {
        // Rows and column chunks wholly outside C are skipped warp-uniformly (tcgen05.ld is warp-collective):
        // a tile that overhangs the matrix edge costs only the part that exists.
        const int64_t row0 =
            static_cast<int64_t>(w.tm) * p.tile_m + static_cast<int64_t>(rank) * p.cta_m + h * 128 + q * 32;
        if (row0 >= p.rows_a) break;
        const int64_t row = row0 + lane;
        const int row_local = h * 128 + q * 32 + lane;  // row within this CTA's part of the tile
        if (p.stage_c && !contrib) {
          const uint32_t stg = data + p.epi_stage_off + static_cast<uint32_t>(e) * 4096u;
          const int rows_in = p.rows_a - row0 < 32 ? static_cast<int>(p.rows_a - row0) : 32;
          if (p.out_kind == OUT_F32_PARTIAL) {  // 32 fp32 columns per 128-byte row
            float* ob = static_cast<float*>(p.out) + static_cast<int64_t>(w.split) * p.out_split_stride;
            for (int c = grp; c < nchunks; c += kGroups) {
              const int64_t col0 = static_cast<int64_t>(w.tn) * p.tile_n + c * 32;
              if (col0 >= p.rows_b) break;
              uint32_t v[32];
              if (zero) {
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = 0u;
              } else {
                tmem_ld_32cols(tmem_base + acc * p.acc_cols + h * p.tile_n + c * 32 + (static_cast<uint32_t>(q * 32) << 16),
                               v);
                tmem_ld_wait();
              }
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {
                uint4 pc[4];
#pragma unroll
                for (int k4 = 0; k4 < 4; ++k4)
                  pc[k4] = make_uint4(v[16 * hh + 4 * k4], v[16 * hh + 4 * k4 + 1], v[16 * hh + 4 * k4 + 2],
                                      v[16 * hh + 4 * k4 + 3]);
                stage_write4(stg, lane, 4 * hh, pc);
              }
              stage_flush(stg, lane, reinterpret_cast<uint8_t*>(ob + row0 * p.out_si + col0), p.out_si * 4, rows_in,
                          (p.rows_b - col0) / 4 < 8 ? static_cast<int>((p.rows_b - col0) / 4) : 8);
            }
          } else {  // 64 half-precision columns (two TMEM chunks) per 128-byte row
            const int bf = p.out_kind == OUT_BF16;
            uint16_t* ob = static_cast<uint16_t*>(p.out);
            for (int c2 = grp; 2 * c2 < nchunks; c2 += kGroups) {
              const int64_t col0 = static_cast<int64_t>(w.tn) * p.tile_n + c2 * 64;
              if (col0 >= p.rows_b) break;
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {
                uint32_t v[32];
                if (zero) {
#pragma unroll
                  for (int j = 0; j < 32; ++j) v[j] = 0u;
                } else {
                  tmem_ld_32cols(tmem_base + acc * p.acc_cols + h * p.tile_n + c2 * 64 + hh * 32 +
                                     (static_cast<uint32_t>(q * 32) << 16),
                                 v);
                  tmem_ld_wait();
                }
                if (owner) add_partials(v, 2 * c2 + hh, row_local, 32, first_unit + 1, j_end);
                uint4 pc[4];
#pragma unroll
                for (int k4 = 0; k4 < 4; ++k4) {
                  pc[k4].x = cvt_pair(__uint_as_float(v[8 * k4 + 0]), __uint_as_float(v[8 * k4 + 1]), bf);
                  pc[k4].y = cvt_pair(__uint_as_float(v[8 * k4 + 2]), __uint_as_float(v[8 * k4 + 3]), bf);
                  pc[k4].z = cvt_pair(__uint_as_float(v[8 * k4 + 4]), __uint_as_float(v[8 * k4 + 5]), bf);
                  pc[k4].w = cvt_pair(__uint_as_float(v[8 * k4 + 6]), __uint_as_float(v[8 * k4 + 7]), bf);
                }
                stage_write4(stg, lane, 4 * hh, pc);
              }
              stage_flush(stg, lane, reinterpret_cast<uint8_t*>(ob + row0 * p.out_si + col0), p.out_si * 2, rows_in,
                          (p.rows_b - col0) / 8 < 8 ? static_cast<int>((p.rows_b - col0) / 8) : 8);
            }
          }
          continue;
        }
        for (int c = grp; c < nchunks; c += kGroups) {
          if (static_cast<int64_t>(w.tn) * p.tile_n + c * 32 >= p.rows_b) break;
          const int ncol = min(32, p.tile_n - c * 32);
          uint32_t v[32];
          if (zero) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0u;
          } else {
            const uint32_t taddr =
                tmem_base + acc * p.acc_cols + h * p.tile_n + c * 32 + (static_cast<uint32_t>(q * 32) << 16);
            if (ncol == 32) {
              tmem_ld_32cols(taddr, v);
            } else {
              tmem_ld_16cols(taddr, v);
            }
            tmem_ld_wait();
          }
          if (contrib) {
            float4* slots4 = reinterpret_cast<float4*>(p.sk_slots);
            const int64_t slot = static_cast<int64_t>(blockIdx.x);
#pragma unroll
            for (int k4 = 0; k4 < 8; ++k4) {
              if (k4 * 4 < ncol)
                slots4[slot_piece(slot, c * 8 + k4, row_local)] =
                    make_float4(__uint_as_float(v[4 * k4]), __uint_as_float(v[4 * k4 + 1]),
                                __uint_as_float(v[4 * k4 + 2]), __uint_as_float(v[4 * k4 + 3]));
            }
            continue;
          }
          if (owner) add_partials(v, c, row_local, ncol, first_unit + 1, j_end);  // contributors' partials, K order
          store_chunk(p, w.split, row, static_cast<int64_t>(w.tn) * p.tile_n + c * 32, ncol, v);
        }
      }
      if (contrib) {  // publish the partial: every thread's stores, then one release of the flag
        __threadfence();
        if (epilogue_sync() && epi_tid == 0) flag_release(p.sk_flags + blockIdx.x, 1);
      } else if (owner) {  // every partial has been read: lower the contributors' flags for the next launch
        if (epilogue_sync() && epi_tid == 0)
          for (int j = first_unit + 1; j < j_end; ++j)
            flag_release(p.sk_flags + (PAIR ? 2 * j + static_cast<int>(rank) : j), 0);
      }
      if (!zero) {
        tc_fence_before();
        if (PAIR) mbar_arrive_cluster(tempty_leader + 8 * acc);
        else mbar_arrive(ctl + OFF_TEMPTY + 8 * acc);
        if (++acc == p.num_acc) {
          acc = 0;
          acc_ph ^= 1u;
        }
      }
    }
    }
  }

  if constexpr (LEAN) {
    if (p.red_cluster) {
      // Every CTA of the cluster holds its partial: CTA r sums its share of the tile over all of them, in split order
      // (0 + p0 + p1 + ...: the order, and so the bits, of the separate reduce kernel), converts and writes C. The
      // second cluster barrier keeps each CTA's shared memory alive until its peers have read it. Every thread of
      // every CTA reaches both barriers, also after a timed-out wait (then the status word holds the error).
      __syncwarp();
      cluster_sync();
      if (warp >= 2) {
        const int S = p.split_k;
        const int r = static_cast<int>(cluster_ctarank());
        const int rows = p.tile_m, cols = p.tile_n;
        const int per = p.red_imajor ? rows / 8 : cols / 8;  // 8-element groups along C's contiguous direction
        const int groups = (p.red_imajor ? cols : rows) * per;
        const int g0 = static_cast<int>(static_cast<int64_t>(groups) * r / S);
        const int g1 = static_cast<int>(static_cast<int64_t>(groups) * (r + 1) / S);
        const Unit w = decode_unit(p, first_unit);
        const int bf = p.out_kind == OUT_BF16;
        uint16_t* out = static_cast<uint16_t*>(p.out);
        for (int g = g0 + static_cast<int>(threadIdx.x) - 64; g < g1; g += EPI_WARPS * 32) {
          int i0, j0;
          uint32_t off;  // float offset of the group in every CTA's partial
          if (p.red_imajor) {
            j0 = g / per;
            i0 = (g - j0 * per) * 8;
            off = static_cast<uint32_t>(j0 * (rows + 4) + i0);
          } else {
            i0 = g / per;
            j0 = (g - i0 * per) * 8;
            off = static_cast<uint32_t>(i0 * (cols + 4) + j0);
          }
          const int64_t gi = static_cast<int64_t>(w.tm) * p.tile_m + i0;
          const int64_t gj = static_cast<int64_t>(w.tn) * p.tile_n + j0;
          if (gi >= p.rows_a || gj >= p.rows_b) continue;
          float4 xa[8], xb[8];  // every split's 8 values in flight before the ordered additions
#pragma unroll
          for (int sp = 0; sp < 8; ++sp) {
            if (sp < S) {
              const uint32_t a = map_to_rank(data + off * 4u, static_cast<uint32_t>(sp));
              xa[sp] = ld_cluster_v4(a);
              xb[sp] = ld_cluster_v4(a + 16u);
            }
          }
          float acc8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int sp = 0; sp < 8; ++sp) {
            if (sp < S) {
              acc8[0] += xa[sp].x;
              acc8[1] += xa[sp].y;
              acc8[2] += xa[sp].z;
              acc8[3] += xa[sp].w;
              acc8[4] += xb[sp].x;
              acc8[5] += xb[sp].y;
              acc8[6] += xb[sp].z;
              acc8[7] += xb[sp].w;
            }
          }
          // the group runs along i (red_imajor) or j; elements past C's edge are skipped
          const int64_t lim = p.red_imajor ? p.rows_a - gi : p.rows_b - gj;
          const int64_t step = p.red_imajor ? p.out_si : p.out_sj;
          uint16_t* dst = out + gi * p.out_si + gj * p.out_sj;
          if (lim >= 8 && step == 1 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
            uint4 pk;
            pk.x = cvt_pair(acc8[0], acc8[1], bf);
            pk.y = cvt_pair(acc8[2], acc8[3], bf);
            pk.z = cvt_pair(acc8[4], acc8[5], bf);
            pk.w = cvt_pair(acc8[6], acc8[7], bf);
            *reinterpret_cast<uint4*>(dst) = pk;
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (e < lim) dst[e * step] = cvt_one(acc8[e], bf);
          }
        }
      }
      __syncwarp();
      cluster_sync();
    }
  }

  __syncwarp();
  tc_fence_before();
  if (PAIR) {
    cluster_sync();  // no CTA leaves while its peer may still signal it or read its shared memory
  } else {
    __syncthreads();
  }
  if (warp == 1) {
    tc_fence_after();
    if (PAIR) tmem_dealloc_pair(tmem_base, p.tmem_cols);
    else tmem_dealloc(tmem_base, p.tmem_cols);
  }
}

// dst[o * ld + i] = src[o * s_outer + i * s_inner] for o < outer, i < inner (2-byte elements). Stages an operand TMA
// cannot read in place (unaligned leading dimension or arbitrary strides) into a 16-byte-aligned copy.
__global__ void pack_kernel(const uint16_t* __restrict__ src, int64_t s_outer, int64_t s_inner,
                            uint16_t* __restrict__ dst, int64_t ld, int64_t outer, int64_t inner) {
  const int64_t total = outer * inner;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t o = idx / inner;
    const int64_t i = idx - o * inner;
    dst[o * ld + i] = src[o * s_outer + i * s_inner];
  }
}

// C[m, n] = cast(sum_{s < split} ws[s, m, n]) in increasing s (the reference's fixed-order reduce,
// kernels/triton_matmul.py:85-92). vec: N % 4 == 0, scn == 1, scm % 4 == 0 and C 8-byte aligned.
// The loads of four splits are issued before their additions (the additions keep increasing s, so the sum is the
// same bit for bit): a thread's time is about split / 4 memory latencies, not split of them. With the few threads a
// decode GEMM's output needs, that latency chain is the whole kernel.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, void* __restrict__ C, int64_t M, int64_t N,
                                     int64_t scm, int64_t scn, int split, int bf16, int vec) {
  // Launched as a programmatic dependent of the GEMM (its launch overlaps the GEMM's tail): wait until the GEMM
  // grid has completed and its partials are visible. Without that launch attribute this returns at once.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t MN = M * N;
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  uint16_t* c = static_cast<uint16_t*>(C);
  if (vec) {
    const float4* w4 = reinterpret_cast<const float4*>(ws);
    const int64_t mn4 = MN / 4;
    for (int64_t q = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; q < mn4; q += step) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      int s = 0;
      for (; s + 4 <= split; s += 4) {
        float4 x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) x[u] = w4[(s + u) * mn4 + q];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          acc.x += x[u].x;
          acc.y += x[u].y;
          acc.z += x[u].z;
          acc.w += x[u].w;
        }
      }
      for (; s < split; ++s) {
        const float4 x = w4[s * mn4 + q];
        acc.x += x.x;
        acc.y += x.y;
        acc.z += x.z;
        acc.w += x.w;
      }
      const int64_t idx = q * 4;
      const int64_t m = idx / N;
      const int64_t n = idx - m * N;
      uint2 w;
      w.x = cvt_pair(acc.x, acc.y, bf16);
      w.y = cvt_pair(acc.z, acc.w, bf16);
      *reinterpret_cast<uint2*>(c + m * scm + n) = w;
    }
    return;
  }
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < MN; idx += step) {
    float acc = 0.f;
    int s = 0;
    for (; s + 4 <= split; s += 4) {
      float x[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) x[u] = ws[(s + u) * MN + idx];
#pragma unroll
      for (int u = 0; u < 4; ++u) acc += x[u];
    }
    for (; s < split; ++s) acc += ws[s * MN + idx];
    const int64_t m = idx / N;
    const int64_t n = idx - m * N;
    c[m * scm + n * scn] = cvt_one(acc, bf16);
  }
}

}  // namespace b2g

// =====================================================================================================================
// host side
// =====================================================================================================================
using namespace b2g;

namespace {
thread_local std::string g_last_error;
}  // namespace

namespace b2g {
// The message b2g_last_error() returns on this thread (the timing helpers in b2g_timing.cu report through it too).
int32_t record_error(int32_t code, const std::string& msg) {
  g_last_error = msg;
  return code;
}
}  // namespace b2g

namespace {

int32_t fail(int32_t code, const std::string& msg) { return record_error(code, msg); }

int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn(std::string& err) {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  static std::string once_err;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr) {
      once_err = std::string("cuTensorMapEncodeTiled unavailable: ") + cudaGetErrorString(e);
      return;
    }
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  err = once_err;
  return fn;
}

// One operand of the MMA: element (r, k) at ptr + r*s_r + k*s_k, r < rows (the MN side), k < K.
struct Operand {
  const void* src;
  int64_t rows, K, s_r, s_k;
  int tile_rows;
  // decided layout
  int mn_major;
  int pack;
  int64_t ld;   // elements between rows (K-major) or between k (MN-major) of what TMA reads
  size_t ws_off;  // where the packed copy lives in the workspace
};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Decide how TMA reads an operand: in place (K-major or MN-major) or through a packed, 16-byte-strided copy.
void layout_operand(Operand& o) {
  int64_t s_r = o.s_r, s_k = o.s_k;
  if (o.K == 1) s_k = 1;
  if (o.rows == 1 && s_k != 1) s_r = 1;
  const bool mn_ok = (o.tile_rows % 64) == 0;
  o.pack = 0;
  if (s_k == 1) {
    const int64_t ld = (o.rows == 1) ? round_up(o.K, 8) : s_r;
    if (aligned16(o.src) && ld >= o.K && (ld % 8) == 0 && ld < (int64_t(1) << 39)) {
      o.mn_major = 0;
      o.ld = ld;
      return;
    }
  }
  if (s_r == 1 && mn_ok) {
    const int64_t ld = (o.K == 1) ? round_up(o.rows, 8) : s_k;
    if (aligned16(o.src) && ld >= o.rows && (ld % 8) == 0 && ld < (int64_t(1) << 39)) {
      o.mn_major = 1;
      o.ld = ld;
      return;
    }
  }
  o.pack = 1;
  if (s_r == 1 && mn_ok) {  // coalesced copy keeping the MN-contiguous layout
    o.mn_major = 1;
    o.ld = round_up(o.rows, 8);
  } else {
    o.mn_major = 0;
    o.ld = round_up(o.K, 8);
  }
}

size_t packed_bytes(const Operand& o) {
  if (!o.pack) return 0;
  const int64_t outer = o.mn_major ? o.K : o.rows;
  return static_cast<size_t>(round_up(outer * o.ld * 2, 256));
}

struct Geometry {
  bool swapped;
  int pair;
  int tile_m, tile_n, bk, stages, epi_warps;
  int cta_m, cta_n;
  int tiles_m, tiles_n, num_kb, units;
  uint32_t acc_cols, num_acc, tmem_cols;
  size_t smem;
  Operand a, b;  // MMA "A" (rows over tile_m) and MMA "B" (rows over tile_n)
  size_t ws_partial;  // split-K partial bytes
  int streamk;
  int64_t sk_iters;     // tiles * num_kb
  int64_t sk_max_ctas;  // upper bound on resident CTAs (sizes the fix-up slots)
  size_t sk_flags_off, sk_slots_off;
  size_t ws_total;
  int red_cluster;  // split-K summed in a cluster of the tile's CTAs through shared memory: no partials in the workspace
};

uint32_t pow2_at_least(uint32_t x) {
  uint32_t p = 32;
  while (p < x) p <<= 1;
  return p;
}

int32_t init_device(int dev, int& sm_count);

// A launch with the in-cluster split-K sum asks for at least this much shared memory, so one CTA runs per SM: the
// CTAs of a cluster then sit on distinct SMs and never wait on each other's tensor memory allocation.
constexpr size_t kRedSmemFloor = kMaxSmemPerCta / 2 + 1024;
// Clusters of 1..8 such CTAs that a B200 holds at once (cudaOccupancyMaxActiveClusters; used when no device is current)
constexpr int kB200Clusters[9] = {0, 148, 74, 45, 33, 26, 22, 15, 15};

// How many clusters of `size` CTAs of the lean kernel (E epilogue warps, one CTA per SM) fit on the current device at
// once. Clusters live within a GPC, so this is below SMs / size (45 clusters of 3, 15 of 8 on a B200); a launch that
// needs more runs a second wave of clusters, slower than the reduce kernel it replaces.
int max_active_clusters(int epi_warps, int size) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return kB200Clusters[size];
  }
  static std::mutex mu;
  static int cache[64][2][9];
  static bool filled[64][2][9];
  const int ei = epi_warps == 8 ? 1 : 0;
  std::lock_guard<std::mutex> lock(mu);
  if (!filled[dev][ei][size]) {
    int sms = 0, n = 0;
    if (init_device(dev, sms) == B2G_OK) {
      cudaLaunchConfig_t lc = {};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = static_cast<unsigned>(size);
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      lc.gridDim = dim3(static_cast<unsigned>(size), 1, 1);
      lc.blockDim = dim3((2 + epi_warps) * 32, 1, 1);
      lc.dynamicSmemBytes = kRedSmemFloor;
      lc.attrs = attr;
      lc.numAttrs = 1;
      const cudaError_t e = ei ? cudaOccupancyMaxActiveClusters(&n, gemm_kernel<8, 0, 1>, &lc)
                               : cudaOccupancyMaxActiveClusters(&n, gemm_kernel<4, 0, 1>, &lc);
      if (e != cudaSuccess) {
        cudaGetLastError();
        n = 0;
      }
    }
    cache[dev][ei][size] = n;
    filled[dev][ei][size] = true;
  }
  return cache[dev][ei][size];
}

// allow_red: whether SPLIT_K may be summed inside a cluster (the allocation-free entry point keeps the workspace path).
int32_t make_geometry(const b2g_config* cfg, const b2g_problem* pr, Geometry& g, const void* A, const void* B,
                      bool allow_red = true) {
  if (!cfg || !pr) return fail(B2G_ERR_INVALID_ARG, "null config or problem");
  if (pr->dtype != B2G_DTYPE_F16 && pr->dtype != B2G_DTYPE_BF16)
    return fail(B2G_ERR_INVALID_ARG, "dtype must be B2G_DTYPE_F16 or B2G_DTYPE_BF16");
  if (pr->M < 0 || pr->N < 0 || pr->K < 0) return fail(B2G_ERR_INVALID_ARG, "negative dimension");
  if (pr->M >= (int64_t(1) << 31) || pr->N >= (int64_t(1) << 31) || pr->K >= (int64_t(1) << 31))
    return fail(B2G_ERR_UNSUPPORTED, "dimension_too_large: each of M, N, K must be < 2^31");
  const int bm = cfg->block_m, bn = cfg->block_n, bk = cfg->block_k;
  if (cfg->cluster != 0 && cfg->cluster != 1 && cfg->cluster != 2)
    return fail(B2G_ERR_UNSUPPORTED, "cluster_invalid: cluster must be 1 or 2");
  g.pair = cfg->cluster == 2;
  g.swapped = bm <= 64;
  if (g.swapped) {
    if (bm != 16 && bm != 32 && bm != 48 && bm != 64)
      return fail(B2G_ERR_UNSUPPORTED, "block_m_invalid: skinny BLOCK_M must be 16, 32, 48 or 64");
    if (bn != 128 && bn != 256)
      return fail(B2G_ERR_UNSUPPORTED, "block_n_invalid: BLOCK_M <= 64 needs BLOCK_N 128 or 256");
    if (g.pair && bn != 256)
      return fail(B2G_ERR_UNSUPPORTED, "cluster_tile_invalid: a CTA pair in the skinny form needs BLOCK_N 256");
    g.tile_m = bn;
    g.tile_n = bm;
  } else {
    if (bm != 128 && bm != 256) return fail(B2G_ERR_UNSUPPORTED, "block_m_invalid: BLOCK_M must be <= 64, 128 or 256");
    if (bn < 16 || bn > 256 || bn % 16 != 0)
      return fail(B2G_ERR_UNSUPPORTED, "block_n_invalid: BLOCK_N must be a multiple of 16 in [16, 256]");
    if (g.pair && bm != 256)
      return fail(B2G_ERR_UNSUPPORTED, "cluster_tile_invalid: a CTA pair needs BLOCK_M 256");
    g.tile_m = bm;
    g.tile_n = bn;
  }
  if (g.pair && (g.tile_n % 16 != 0 || (g.tile_n / 2) % 8 != 0))
    return fail(B2G_ERR_UNSUPPORTED, "cluster_tile_invalid: each CTA of a pair needs a multiple of 8 B rows");
  g.cta_m = g.pair ? g.tile_m / 2 : g.tile_m;
  g.cta_n = g.pair ? g.tile_n / 2 : g.tile_n;
  if (bk != 64 && bk != 128) return fail(B2G_ERR_UNSUPPORTED, "block_k_invalid: BLOCK_K must be 64 or 128");
  if (cfg->num_warps != 4 && cfg->num_warps != 8)
    return fail(B2G_ERR_UNSUPPORTED, "num_warps_invalid: epilogue warps must be 4 or 8");
  if (cfg->num_stages < 2 || cfg->num_stages > kMaxStages)
    return fail(B2G_ERR_UNSUPPORTED, "num_stages_invalid: stages must be in [2, 16]");
  if (cfg->group_m < 1) return fail(B2G_ERR_UNSUPPORTED, "group_m_invalid: GROUP_M must be >= 1");
  if (cfg->split_k < 1 || cfg->split_k > 64) return fail(B2G_ERR_UNSUPPORTED, "split_k_invalid: SPLIT_K in [1, 64]");
  if (cfg->schedule != B2G_SCHED_PERSISTENT && cfg->schedule != B2G_SCHED_TILE &&
      cfg->schedule != B2G_SCHED_STREAMK)
    return fail(B2G_ERR_UNSUPPORTED, "schedule_invalid");
  if (cfg->schedule == B2G_SCHED_STREAMK && cfg->split_k != 1)
    return fail(B2G_ERR_UNSUPPORTED, "streamk_with_split_k: stream-K balances K itself; SPLIT_K must be 1");
  if (cfg->wait_limit_us < 0) return fail(B2G_ERR_INVALID_ARG, "wait_limit_us must be >= 0");
  if (cfg->wait_limit_us > 0 && g.pair)
    return fail(B2G_ERR_UNSUPPORTED,
                "wait_limit_single_cta_only: a CTA pair keeps the default wait limit (an early stop cannot wait out "
                "the second CTA's copies)");
  g.streamk = cfg->schedule == B2G_SCHED_STREAMK;
  g.bk = bk;
  g.stages = cfg->num_stages;
  g.epi_warps = cfg->num_warps;

  const int64_t M = pr->M, N = pr->N, K = pr->K;
  // operands in MMA orientation
  Operand oa{}, ob{};
  if (!g.swapped) {
    oa = Operand{A, M, K, pr->stride_am, pr->stride_ak, g.cta_m, 0, 0, 0, 0};
    ob = Operand{B, N, K, pr->stride_bn, pr->stride_bk, g.cta_n, 0, 0, 0, 0};
  } else {
    oa = Operand{B, N, K, pr->stride_bn, pr->stride_bk, g.cta_m, 0, 0, 0, 0};
    ob = Operand{A, M, K, pr->stride_am, pr->stride_ak, g.cta_n, 0, 0, 0, 0};
  }
  layout_operand(oa);
  layout_operand(ob);
  g.a = oa;
  g.b = ob;
  const int64_t rows_a = g.swapped ? N : M;
  const int64_t rows_b = g.swapped ? M : N;
  g.tiles_m = static_cast<int>((rows_a + g.tile_m - 1) / g.tile_m);
  g.tiles_n = static_cast<int>((rows_b + g.tile_n - 1) / g.tile_n);
  g.num_kb = static_cast<int>((K + bk - 1) / bk);
  const int64_t units = static_cast<int64_t>(g.tiles_m) * g.tiles_n * cfg->split_k;
  if (units >= (int64_t(1) << 31)) return fail(B2G_ERR_UNSUPPORTED, "too_many_tiles");
  if (static_cast<int64_t>(cfg->split_k) * g.num_kb >= (int64_t(1) << 31))
    return fail(B2G_ERR_UNSUPPORTED, "split_k_too_deep: SPLIT_K x K blocks must be < 2^31");
  g.units = static_cast<int>(units);
  // fp32 accumulator columns per CTA: a pair's CTA holds its 128 rows x tile_n
  g.acc_cols = static_cast<uint32_t>(g.pair ? g.tile_n : g.tile_m / 128 * g.tile_n);
  g.num_acc = (2 * g.acc_cols <= 512) ? 2u : 1u;
  g.tmem_cols = pow2_at_least(g.num_acc * g.acc_cols);
  const size_t stage = static_cast<size_t>(g.cta_m + g.cta_n) * bk * 2;
  g.smem = kCtlBytes + kAlignSlack + stage * g.stages;
  if (g.smem > kMaxSmemPerCta) return fail(B2G_ERR_UNSUPPORTED, "smem_exceeds_limit");
  const int64_t ws_elems = static_cast<int64_t>(cfg->split_k) * M * N;
  if (cfg->split_k > 1 && ws_elems >= (int64_t(1) << 40))
    return fail(B2G_ERR_UNSUPPORTED, "split_k_workspace_too_large");
  g.ws_partial = cfg->split_k > 1 ? static_cast<size_t>(round_up(ws_elems * 4, 256)) : 0;
  size_t sk_bytes = 0;
  g.sk_iters = static_cast<int64_t>(g.tiles_m) * g.tiles_n * g.num_kb;
  g.sk_max_ctas = 0;
  g.sk_flags_off = g.sk_slots_off = 0;
  if (g.streamk) {
    // at most as many resident CTAs as smem and tensor memory allow per SM on every SM
    int sms = kDefaultSmCount;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) {
      int v = 0;
      if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0) sms = v;
    } else {
      cudaGetLastError();
    }
    const int64_t per_sm = std::max<int64_t>(
        1, std::min<int64_t>(static_cast<int64_t>(kMaxSmemPerCta / g.smem), 512 / static_cast<int64_t>(g.tmem_cols)));
    g.sk_max_ctas = static_cast<int64_t>(sms) * per_sm;
    g.sk_flags_off = 0;  // flags first: the caller zeroes them once, the kernels leave them zero
    g.sk_slots_off = static_cast<size_t>(round_up(g.sk_max_ctas * 4, 256));
    sk_bytes = g.sk_slots_off +
               static_cast<size_t>(round_up(g.sk_max_ctas * static_cast<int64_t>(g.cta_m) * g.tile_n * 4, 256));
  }
  if (K == 0) {
    // An empty K only zero-fills C: no GEMM launch, so no partials, fix-up state or staged operands are needed.
    g.ws_partial = 0;
    sk_bytes = 0;
    g.a.pack = g.b.pack = 0;
  }
  // SPLIT_K of 2..8 on single-CTA tiles of at most 8192 outputs is summed inside a cluster of the tile's CTAs when
  // every cluster of the launch fits on the GPU at once (one CTA per unit, one wave): each CTA keeps its fp32 partial in its own operand
  // ring (free once the tile's MMAs are done) and the sum reads the peers' rings. Same split order as the reduce
  // kernel, so the same bits, without the second launch or the partials' round trip through global memory.
  g.red_cluster = 0;
  if (allow_red && K > 0 && cfg->split_k >= 2 && cfg->split_k <= kMaxRedCluster && !g.pair && !g.streamk) {
    const size_t red_bytes = static_cast<size_t>(g.tile_m + 4) * (g.tile_n + 4) * 4;
    const size_t ring = stage * g.stages;
    const int64_t clusters = static_cast<int64_t>(g.tiles_m) * g.tiles_n;
    // Larger partials (128 x 128 tiles: 64 KB per CTA) measured 4-5 % slower summed this way than by the reduce
    // kernel spread over every SM; decode-shaped and 128 x 64 tiles 3-16 % faster.
    const bool small = static_cast<int64_t>(g.tile_m) * g.tile_n <= kMaxRedElems;
    if (small && red_bytes <= ring && clusters <= max_active_clusters(g.epi_warps, cfg->split_k)) {
      g.red_cluster = 1;
      g.ws_partial = 0;
    }
  }
  // workspace: [split-K partials][stream-K flags + slots][staged A][staged B]
  g.sk_flags_off += g.ws_partial;
  g.sk_slots_off += g.ws_partial;
  g.a.ws_off = g.ws_partial + sk_bytes;
  g.b.ws_off = g.a.ws_off + packed_bytes(g.a);
  g.ws_total = g.b.ws_off + packed_bytes(g.b);
  return B2G_OK;
}

struct DeviceInit {
  std::once_flag flag;
  cudaError_t err = cudaSuccess;
  int sm_count = 0;
};
DeviceInit g_dev[64];

int32_t init_device(int dev, int& sm_count) {
  if (dev < 0 || dev >= 64) return fail(B2G_ERR_CUDA, "device index out of range");
  DeviceInit& d = g_dev[dev];
  std::call_once(d.flag, [&d, dev] {
    const int smem = static_cast<int>(kMaxSmemPerCta);
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel<4, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(gemm_kernel<8, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(gemm_kernel<4, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(gemm_kernel<8, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(gemm_kernel<4, 0, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(gemm_kernel<8, 0, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    // a pair is a 2-CTA cluster: always within the portable size, no opt-in needed
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev);
    d.err = e;
  });
  if (d.err != cudaSuccess) return fail(B2G_ERR_CUDA, std::string("device set-up: ") + cudaGetErrorString(d.err));
  sm_count = d.sm_count;
  return B2G_OK;
}

int32_t encode_operand(const Operand& o, const void* base, int dtype, int bk, CUtensorMap* map, int32_t* is3d) {
  std::string err;
  EncodeTiledFn enc = get_encode_fn(err);
  if (!enc) return fail(B2G_ERR_CUDA, err);
  const CUtensorMapDataType dt = dtype == B2G_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  *is3d = 0;
  // An MN-major operand whose rows are whole 64-wide groups is described as (64 rows, K, row groups), so one copy
  // per K block fetches every group a CTA needs. The groups never reach past the last row, so nothing outside the
  // matrix is read. If the driver declines the shape, the 2-D description below is used.
  if (o.mn_major && o.tile_rows > 64 && o.tile_rows % 64 == 0 && o.rows % 64 == 0) {
    cuuint64_t dims3[3] = {64, static_cast<cuuint64_t>(o.K), static_cast<cuuint64_t>(o.rows / 64)};
    cuuint64_t strides3[2] = {static_cast<cuuint64_t>(o.ld) * 2, 128};
    cuuint32_t box3[3] = {64, static_cast<cuuint32_t>(bk), static_cast<cuuint32_t>(o.tile_rows / 64)};
    cuuint32_t estr3[3] = {1, 1, 1};
    if (enc(map, dt, 3, const_cast<void*>(base), dims3, strides3, box3, estr3, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS) {
      *is3d = 1;
      return B2G_OK;
    }
  }
  cuuint64_t dims[2];
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(o.ld) * 2};
  cuuint32_t box[2];
  cuuint32_t estr[2] = {1, 1};
  if (o.mn_major) {
    dims[0] = static_cast<cuuint64_t>(o.rows);
    dims[1] = static_cast<cuuint64_t>(o.K);
    box[0] = 64;
    box[1] = static_cast<cuuint32_t>(bk);
  } else {
    dims[0] = static_cast<cuuint64_t>(o.K);
    dims[1] = static_cast<cuuint64_t>(o.rows);
    box[0] = 64;
    box[1] = static_cast<cuuint32_t>(o.tile_rows);
  }
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[256];
    snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu, ld %lld, box %u x %u", (int)r,
             (unsigned long long)dims[0], (unsigned long long)dims[1], (long long)o.ld, box[0], box[1]);
    return fail(B2G_ERR_CUDA, buf);
  }
  return B2G_OK;
}

}  // namespace

struct b2g_plan {
  int device;
  int empty;       // M == 0 or N == 0: nothing to launch
  int k_zero;      // K == 0: only the zero fill
  KParams kp;
  CUtensorMap tma_a, tma_b;
  int epi_warps;
  int pair;
  int lean;        // one CTA per unit, no stream-K or in-kernel split-K sum: the lean kernel form
  int grid, threads;
  size_t smem;
  // packing
  int pack_a, pack_b;
  const void* pa_src;
  int64_t pa_so, pa_si, pa_ld, pa_outer, pa_inner;
  void* pa_dst;
  const void* pb_src;
  int64_t pb_so, pb_si, pb_ld, pb_outer, pb_inner;
  void* pb_dst;
  // split-K reduce
  int reduce;
  const float* r_ws;
  void* r_c;
  int64_t r_M, r_N, r_scm, r_scn;
  int r_split, r_bf16, r_vec;
  // what b2g_plan_rebind needs: the caller's pointers, the MMA operands' layouts (MMA "A" is the caller's B when
  // `swapped`), the element type and K step
  const void* user_a;
  const void* user_b;
  void* user_c;
  Operand op_a, op_b;
  int swapped, dtype, bk;
};

namespace {

void fill_pack(const Operand& o, void* ws, const void*& src, int64_t& so, int64_t& si, int64_t& ld, int64_t& outer,
               int64_t& inner, void*& dst) {
  src = o.src;
  dst = static_cast<uint8_t*>(ws) + o.ws_off;
  ld = o.ld;
  if (o.mn_major) {
    outer = o.K;
    inner = o.rows;
    so = o.s_k;
    si = o.s_r;
  } else {
    outer = o.rows;
    inner = o.K;
    so = o.s_r;
    si = o.s_k;
  }
}

int grid_for(int64_t work, int per_block) {
  int64_t g = (work + per_block - 1) / per_block;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(g, 148 * 16)));
}

// Fill `p` (caller-owned) with the launch plan of (cfg, prob) on the current device.
int32_t plan_init(b2g_plan* p, const b2g_config* cfg, const b2g_problem* prob, const void* A, const void* B, void* C,
                  void* workspace, size_t workspace_bytes, int32_t* status, bool allow_red = true) {
  Geometry g;
  int32_t rc = make_geometry(cfg, prob, g, A, B, allow_red);
  if (rc != B2G_OK) return rc;
  const int64_t M = prob->M, N = prob->N, K = prob->K;
  if ((M > 0 && N > 0) && (!C || (K > 0 && (!A || !B)))) return fail(B2G_ERR_INVALID_ARG, "null A, B or C");
  if (g.ws_total > 0 && (workspace == nullptr || workspace_bytes < g.ws_total)) {
    char buf[160];
    snprintf(buf, sizeof buf, "workspace of %zu bytes needed, %zu given", g.ws_total,
             workspace == nullptr ? size_t(0) : workspace_bytes);
    return fail(B2G_ERR_WORKSPACE, buf);
  }
  if (g.ws_total > 0 && (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(B2G_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return fail(B2G_ERR_CUDA, cudaGetErrorString(ce));
  int sm_count = 0;
  rc = init_device(dev, sm_count);
  if (rc != B2G_OK) return rc;

  memset(p, 0, sizeof(*p));
  p->device = dev;
  p->empty = (M == 0 || N == 0);
  p->k_zero = (K == 0);
  const int bf16 = prob->dtype == B2G_DTYPE_BF16;
  if (!p->empty && p->k_zero) {
    p->reduce = 1;
    p->r_ws = nullptr;
    p->r_c = C;
    p->r_M = M;
    p->r_N = N;
    p->r_scm = prob->stride_cm;
    p->r_scn = prob->stride_cn;
    p->r_split = 0;
    p->r_bf16 = bf16;
    p->r_vec = 0;
  }
  if (!p->empty && !p->k_zero) {
    const void* a_base = g.a.src;
    const void* b_base = g.b.src;
    if (g.a.pack) {
      p->pack_a = 1;
      fill_pack(g.a, workspace, p->pa_src, p->pa_so, p->pa_si, p->pa_ld, p->pa_outer, p->pa_inner, p->pa_dst);
      a_base = p->pa_dst;
    }
    if (g.b.pack) {
      p->pack_b = 1;
      fill_pack(g.b, workspace, p->pb_src, p->pb_so, p->pb_si, p->pb_ld, p->pb_outer, p->pb_inner, p->pb_dst);
      b_base = p->pb_dst;
    }
    KParams& k = p->kp;
    rc = encode_operand(g.a, a_base, prob->dtype, g.bk, &p->tma_a, &k.a_3d);
    if (rc == B2G_OK) rc = encode_operand(g.b, b_base, prob->dtype, g.bk, &p->tma_b, &k.b_3d);
    if (rc != B2G_OK) return rc;
    k.rows_a = static_cast<int32_t>(g.swapped ? N : M);
    k.rows_b = static_cast<int32_t>(g.swapped ? M : N);
    k.K = static_cast<int32_t>(K);
    k.tile_m = g.tile_m;
    k.tile_n = g.tile_n;
    k.cta_m = g.cta_m;
    k.cta_n = g.cta_n;
    k.bk = g.bk;
    k.stages = g.stages;
    // a group taller than the matrix is one group of all tile rows: same order, and the divisors stay small
    k.group_m = std::max(1, std::min(cfg->group_m, g.tiles_m));
    k.split_k = cfg->split_k;
    {
      const int gm = k.group_m;
      const int last_first = ((g.tiles_m - 1) / gm) * gm;
      k.fd_split = make_fastdiv(static_cast<uint32_t>(std::max(1, cfg->split_k)));
      k.fd_group = make_fastdiv(static_cast<uint32_t>(gm) * static_cast<uint32_t>(g.tiles_n));
      k.fd_gm = make_fastdiv(static_cast<uint32_t>(gm));
      k.fd_last = make_fastdiv(static_cast<uint32_t>(std::min(gm, g.tiles_m - last_first)));
      k.last_group_first = last_first;
    }
    k.tiles_m = g.tiles_m;
    k.tiles_n = g.tiles_n;
    k.num_kb = g.num_kb;
    k.units = g.units;
    k.a_mn_major = g.a.mn_major;
    k.b_mn_major = g.b.mn_major;
    k.idesc = idesc_f16(bf16 ? 1u : 0u, static_cast<uint32_t>(g.a.mn_major), static_cast<uint32_t>(g.b.mn_major),
                        g.pair ? 256u : 128u, static_cast<uint32_t>(g.tile_n));
    k.a_stage_bytes = static_cast<uint32_t>(g.cta_m * g.bk * 2);
    k.b_stage_bytes = static_cast<uint32_t>(g.cta_n * g.bk * 2);
    k.acc_cols = g.acc_cols;
    k.num_acc = g.num_acc;
    k.tmem_cols = g.tmem_cols;
    k.status = status;
    k.timeout_ns = cfg->wait_limit_us > 0 ? static_cast<uint64_t>(cfg->wait_limit_us) * 1000ull : kWaitTimeoutNs;
    k.streamk = g.streamk;
    k.sk_dp_tiles = 0;
    k.sk_workers = 1;
    k.sk_iters = g.sk_iters;
    k.sk_flags = g.streamk ? reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + g.sk_flags_off) : nullptr;
    k.sk_slots = g.streamk ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + g.sk_slots_off) : nullptr;
    k.red_cluster = g.red_cluster;
    if (cfg->split_k > 1 && !g.red_cluster) {
      k.out = workspace;
      k.out_kind = OUT_F32_PARTIAL;
      k.out_split_stride = M * N;
      k.out_si = g.swapped ? 1 : N;
      k.out_sj = g.swapped ? N : 1;
      k.vec_ok = (k.out_sj == 1) && (k.out_si % 4 == 0);
      p->reduce = 1;
      p->r_ws = static_cast<const float*>(workspace);
      p->r_c = C;
      p->r_M = M;
      p->r_N = N;
      p->r_scm = prob->stride_cm;
      p->r_scn = prob->stride_cn;
      p->r_split = cfg->split_k;
      p->r_bf16 = bf16;
      p->r_vec = (N % 4 == 0) && prob->stride_cn == 1 && (prob->stride_cm % 4 == 0) &&
                 ((reinterpret_cast<uintptr_t>(C) & 7u) == 0);
    } else {
      k.out = C;
      k.out_kind = bf16 ? OUT_BF16 : OUT_F16;
      k.out_split_stride = 0;
      k.out_si = g.swapped ? prob->stride_cn : prob->stride_cm;
      k.out_sj = g.swapped ? prob->stride_cm : prob->stride_cn;
      k.vec_ok = (k.out_sj == 1) && (k.out_si % 8 == 0) && ((reinterpret_cast<uintptr_t>(C) & 15u) == 0);
      // the cluster sum writes 8 outputs at a time along C's contiguous direction
      k.red_imajor = (k.out_sj != 1 && k.out_si == 1) ? 1 : 0;
    }
    p->epi_warps = g.epi_warps;
    p->pair = g.pair;
    p->threads = (2 + g.epi_warps) * 32;
    p->smem = g.red_cluster ? std::max(g.smem, kRedSmemFloor) : g.smem;
    {
      // staged epilogue: row-major C (or the fp32 partials) in whole 16-byte pieces, 64-column half-precision chunk
      // pairs, and room for 4 KB per epilogue warp next to the ring
      const size_t staging = static_cast<size_t>(g.epi_warps) * 4096;
      const bool partial = cfg->split_k > 1;
      const bool pieces_ok = partial ? (N % 4 == 0) : (N % 8 == 0 && g.tile_n % 64 == 0);
      if (!g.swapped && !g.red_cluster && k.vec_ok && pieces_ok && g.smem + staging <= kMaxSmemPerCta) {
        k.stage_c = 1;
        k.epi_stage_off = static_cast<uint32_t>(static_cast<size_t>(g.cta_m + g.cta_n) * g.bk * 2 * g.stages);
        p->smem = g.smem + staging;
      }
    }
    // grid in work units (CTAs, or CTA pairs)
    int64_t grid = g.units;
    if (cfg->schedule == B2G_SCHED_PERSISTENT || cfg->schedule == B2G_SCHED_STREAMK) {
      int64_t slots = 0;
      if (g.pair) {
        cudaLaunchConfig_t lc = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        lc.gridDim = dim3(2 * sm_count, 1, 1);
        lc.blockDim = dim3(p->threads, 1, 1);
        lc.dynamicSmemBytes = p->smem;
        lc.attrs = attr;
        lc.numAttrs = 1;
        int nclusters = 0;
        ce = (g.epi_warps == 4) ? cudaOccupancyMaxActiveClusters(&nclusters, gemm_kernel<4, 1>, &lc)
                                : cudaOccupancyMaxActiveClusters(&nclusters, gemm_kernel<8, 1>, &lc);
        if (ce != cudaSuccess) return fail(B2G_ERR_CUDA, std::string("cluster occupancy query: ") + cudaGetErrorString(ce));
        slots = std::max(1, nclusters);
      } else {
        int occ = 0;
        ce = (g.epi_warps == 4)
                 ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gemm_kernel<4, 0>, p->threads, p->smem)
                 : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gemm_kernel<8, 0>, p->threads, p->smem);
        if (ce != cudaSuccess) return fail(B2G_ERR_CUDA, std::string("occupancy query: ") + cudaGetErrorString(ce));
        occ = std::max(1, std::min<int>(occ, static_cast<int>(512 / g.tmem_cols)));
        slots = static_cast<int64_t>(sm_count) * occ;
      }
      grid = std::min<int64_t>(grid, slots);
      if (g.streamk) {
        // Every worker resident at once (owners wait for contributors). By the last wave's fill:
        //  * the tiles of the partial last wave (r of them) fit at least twice into the workers: every full wave runs
        //    data-parallel and each of the r tiles is split evenly over s = workers / r workers in K, so the last
        //    wave takes 1/s of a tile's time (plus one fix-up, which overlaps the worker's next tile) instead of a
        //    whole one;
        //  * otherwise (a last wave more than half full, or no partial wave) every tile runs data-parallel: the wave
        //    loses at most half a tile's time, and sharing all tiles' K blocks among the workers (one fix-up per
        //    tile) measured slower than that on B200 (2048^3: 58 against 34 us).
        const int64_t tiles = static_cast<int64_t>(g.tiles_m) * g.tiles_n;
        grid = std::min<int64_t>(slots, std::max<int64_t>(tiles, 1) * g.num_kb);
        if (grid * (g.pair ? 2 : 1) > g.sk_max_ctas) grid = g.sk_max_ctas / (g.pair ? 2 : 1);
        grid = std::max<int64_t>(grid, 1);
        const int64_t min_slice = std::max<int64_t>(4, g.num_kb / 4);
        const int64_t full = tiles / grid, r = tiles % grid;
        const int64_t split = r > 0 ? std::min<int64_t>(grid / r, std::max<int64_t>(1, g.num_kb / min_slice)) : 0;
        int64_t dp_tiles = tiles, workers = 1;  // whole waves, or a last wave more than half full: data-parallel
        if (r > 0 && split >= 2) {
          dp_tiles = full * grid;
          workers = r * split;
        }
        const int64_t iters = (tiles - dp_tiles) * g.num_kb;
        p->kp.sk_dp_tiles = static_cast<int32_t>(dp_tiles);
        p->kp.sk_iters = iters;
        p->kp.sk_workers = static_cast<int32_t>(workers);
        if (dp_tiles == 0) grid = workers;  // no data-parallel wave: idle workers need not launch
      }
    }
    p->grid = static_cast<int>(std::max<int64_t>(grid, 1));
    p->lean = !g.pair && !g.streamk && grid == g.units;
    if (g.red_cluster && !p->lean)
      return fail(B2G_ERR_UNSUPPORTED, "cluster_split_k: the in-cluster split-K sum needs one CTA per (tile, split)");
  }
  p->user_a = A;
  p->user_b = B;
  p->user_c = C;
  p->op_a = g.a;
  p->op_b = g.b;
  p->swapped = g.swapped;
  p->dtype = prob->dtype;
  p->bk = g.bk;
  return B2G_OK;
}

// Same 16-byte (and 8-byte) alignment class: the layout decisions made for the old pointer hold for the new one.
bool same_alignment(const void* x, const void* y) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(x), b = reinterpret_cast<uintptr_t>(y);
  return (a & 15u) == (b & 15u);
}

// ---------------------------------------------------------------- allocation-free entry point
// Some callers may not allocate device memory at all (see b2g_gemm_noalloc in b2g.h). Their split-K partials live
// in this fixed array instead of a caller workspace. It is part of the module image, so every GPU that loads this
// library holds kNoAllocScratchBytes of it until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // 32 MiB: 8M fp32 partials
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

struct ScratchAddress {
  std::once_flag flag;
  cudaError_t err = cudaSuccess;
  void* ptr = nullptr;
};
ScratchAddress g_scratch_address[64];

// Device address of g_noalloc_scratch on `dev` (the current device). In host code the array's name is only a
// host-side handle, so the address is looked up once per device and cached.
int32_t noalloc_scratch(int dev, void*& ptr) {
  if (dev < 0 || dev >= 64) return fail(B2G_ERR_CUDA, "device index out of range");
  ScratchAddress& s = g_scratch_address[dev];
  std::call_once(s.flag, [&s] { s.err = cudaGetSymbolAddress(&s.ptr, g_noalloc_scratch); });
  if (s.err != cudaSuccess || s.ptr == nullptr)
    return fail(B2G_ERR_CUDA, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(s.err));
  ptr = s.ptr;
  return B2G_OK;
}

}  // namespace

extern "C" {

int32_t b2g_abi_version(void) { return B2G_ABI_VERSION; }
const char* b2g_version(void) { return B2G_VERSION_STR; }
const char* b2g_source_hash(void) { return B2G_SOURCE_HASH; }
const char* b2g_last_error(void) { return g_last_error.c_str(); }

const char* b2g_error_string(int32_t code) {
  switch (code) {
    case B2G_OK: return "ok";
    case B2G_ERR_INVALID_ARG: return "invalid argument";
    case B2G_ERR_UNSUPPORTED: return "unsupported configuration";
    case B2G_ERR_WORKSPACE: return "workspace missing or too small";
    case B2G_ERR_CUDA: return "CUDA error";
    default: return "unknown error";
  }
}

const char* b2g_status_string(int32_t status) {
  switch (status) {
    case 0: return "ok";
    case kStatusProducerTimeout: return "device wait timed out in the TMA producer";
    case kStatusMmaTimeout: return "device wait timed out in the MMA issuer";
    case kStatusEpilogueTimeout: return "device wait timed out in the epilogue";
    case kStatusStreamkTimeout: return "stream-K owner timed out waiting for a contributor's partial";
    case 0x201: return "timing gate released by its time limit, not by the host";
    default: return "unknown device status";
  }
}

int32_t b2g_check(const b2g_config* cfg, const b2g_problem* prob, char* reason, size_t reason_len) {
  Geometry g;
  // alignment of the real pointers is unknown here: assume 16-byte aligned bases (packing covers the rest)
  int32_t rc = make_geometry(cfg, prob, g, reinterpret_cast<const void*>(256), reinterpret_cast<const void*>(256));
  if (rc != B2G_OK && reason && reason_len) {
    strncpy(reason, g_last_error.c_str(), reason_len - 1);
    reason[reason_len - 1] = 0;
  } else if (reason && reason_len) {
    reason[0] = 0;
  }
  return rc;
}

int32_t b2g_workspace_size(const b2g_config* cfg, const b2g_problem* prob, const void* A, const void* B,
                           size_t* bytes) {
  if (!bytes) return fail(B2G_ERR_INVALID_ARG, "null bytes");
  Geometry g;
  const void* dflt = reinterpret_cast<const void*>(256);
  int32_t rc = make_geometry(cfg, prob, g, A ? A : dflt, B ? B : dflt);
  if (rc != B2G_OK) return rc;
  *bytes = g.ws_total;
  return B2G_OK;
}

int32_t b2g_smem_bytes(const b2g_config* cfg, const b2g_problem* prob, size_t* bytes) {
  if (!bytes) return fail(B2G_ERR_INVALID_ARG, "null bytes");
  if (!cfg) return fail(B2G_ERR_INVALID_ARG, "null config");
  const bool pair = cfg->cluster == 2;
  const int rows = cfg->block_m + cfg->block_n;  // A rows + B rows of one tile
  const size_t stage = static_cast<size_t>(pair ? rows / 2 : rows) * cfg->block_k * 2;
  (void)prob;
  *bytes = kCtlBytes + kAlignSlack + stage * cfg->num_stages;
  return B2G_OK;
}

int32_t b2g_plan_create(const b2g_config* cfg, const b2g_problem* prob, const void* A, const void* B, void* C,
                        void* workspace, size_t workspace_bytes, int32_t* status, b2g_plan** out) {
  if (!out) return fail(B2G_ERR_INVALID_ARG, "null plan output");
  *out = nullptr;
  b2g_plan* p = new b2g_plan();
  const int32_t rc = plan_init(p, cfg, prob, A, B, C, workspace, workspace_bytes, status);
  if (rc != B2G_OK) {
    delete p;
    return rc;
  }
  *out = p;
  return B2G_OK;
}

int32_t b2g_plan_launch(const b2g_plan* p, void* stream) {
  if (!p) return fail(B2G_ERR_INVALID_ARG, "null plan");
  if (p->empty) return B2G_OK;
  // A plan's tensor maps and buffers live on the device it was made on; launching it while another device is
  // current would run the kernel against memory that device cannot reach.
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess || cur != p->device) {
    char buf[128];
    snprintf(buf, sizeof buf, "plan was made on device %d but device %d is current", p->device, cur);
    return fail(B2G_ERR_INVALID_ARG, buf);
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (p->pack_a) {
    pack_kernel<<<grid_for(p->pa_outer * p->pa_inner, 256), 256, 0, st>>>(
        static_cast<const uint16_t*>(p->pa_src), p->pa_so, p->pa_si, static_cast<uint16_t*>(p->pa_dst), p->pa_ld,
        p->pa_outer, p->pa_inner);
  }
  if (p->pack_b) {
    pack_kernel<<<grid_for(p->pb_outer * p->pb_inner, 256), 256, 0, st>>>(
        static_cast<const uint16_t*>(p->pb_src), p->pb_so, p->pb_si, static_cast<uint16_t*>(p->pb_dst), p->pb_ld,
        p->pb_outer, p->pb_inner);
  }
  if (!p->k_zero) {
    // a programmatic dependent of whatever precedes it on the stream: its prologue overlaps that kernel's tail
    // (the kernel waits for it before touching global memory)
    cudaLaunchConfig_t lc = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.blockDim = dim3(p->threads, 1, 1);
    lc.dynamicSmemBytes = p->smem;
    lc.stream = st;
    lc.attrs = attr;
    cudaError_t le;
    if (p->pair) {
      attr[1].id = cudaLaunchAttributeClusterDimension;
      attr[1].val.clusterDim.x = 2;
      attr[1].val.clusterDim.y = 1;
      attr[1].val.clusterDim.z = 1;
      lc.gridDim = dim3(2 * p->grid, 1, 1);
      lc.numAttrs = 2;
      le = (p->epi_warps == 4) ? cudaLaunchKernelEx(&lc, gemm_kernel<4, 1>, p->kp, p->tma_a, p->tma_b)
                               : cudaLaunchKernelEx(&lc, gemm_kernel<8, 1>, p->kp, p->tma_a, p->tma_b);
    } else {
      lc.gridDim = dim3(p->grid, 1, 1);
      lc.numAttrs = 1;
      if (p->kp.red_cluster) {  // the SPLIT_K CTAs of a tile (consecutive units) form one cluster
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = static_cast<unsigned>(p->kp.split_k);
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        lc.numAttrs = 2;
      }
      if (p->lean)
        le = (p->epi_warps == 4) ? cudaLaunchKernelEx(&lc, gemm_kernel<4, 0, 1>, p->kp, p->tma_a, p->tma_b)
                                 : cudaLaunchKernelEx(&lc, gemm_kernel<8, 0, 1>, p->kp, p->tma_a, p->tma_b);
      else
        le = (p->epi_warps == 4) ? cudaLaunchKernelEx(&lc, gemm_kernel<4, 0>, p->kp, p->tma_a, p->tma_b)
                                 : cudaLaunchKernelEx(&lc, gemm_kernel<8, 0>, p->kp, p->tma_a, p->tma_b);
    }
    if (le != cudaSuccess) {
      cudaGetLastError();  // a refused launch is not sticky: clear it so the next call does not report it again
      return fail(B2G_ERR_CUDA, std::string("GEMM launch: ") + cudaGetErrorString(le));
    }
  }
  if (p->reduce) {
    const int64_t work = p->r_vec ? p->r_M * p->r_N / 4 : p->r_M * p->r_N;
    cudaLaunchConfig_t lc = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.gridDim = dim3(grid_for(work, 256), 1, 1);
    lc.blockDim = dim3(256, 1, 1);
    lc.dynamicSmemBytes = 0;
    lc.stream = st;
    lc.attrs = attr;
    lc.numAttrs = 1;
    cudaError_t le = cudaLaunchKernelEx(&lc, splitk_reduce_kernel, p->r_ws, p->r_c, p->r_M, p->r_N, p->r_scm,
                                        p->r_scn, p->r_split, p->r_bf16, p->r_vec);
    if (le != cudaSuccess) {
      cudaGetLastError();
      return fail(B2G_ERR_CUDA, std::string("reduce launch: ") + cudaGetErrorString(le));
    }
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(B2G_ERR_CUDA, std::string("launch: ") + cudaGetErrorString(e));
  return B2G_OK;
}

int32_t b2g_plan_rebind(b2g_plan* p, const void* A, const void* B, void* C) {
  if (!p) return fail(B2G_ERR_INVALID_ARG, "null plan");
  if (p->empty) return B2G_OK;
  if (!C || (!p->k_zero && (!A || !B))) return fail(B2G_ERR_INVALID_ARG, "null A, B or C");
  if (!same_alignment(A, p->user_a) || !same_alignment(B, p->user_b) || !same_alignment(C, p->user_c))
    return fail(B2G_ERR_INVALID_ARG,
                "rebind_alignment_changed: a pointer's 16-byte alignment differs from the plan's; create a new plan");
  if (p->k_zero) {
    p->r_c = C;
    p->user_c = C;
    return B2G_OK;
  }
  // MMA operand "a" reads the caller's A (or B when swapped); a staged operand keeps its workspace copy and only
  // changes the source of the staging copy
  const void* src_a = p->swapped ? B : A;
  const void* src_b = p->swapped ? A : B;
  const void* old_a = p->swapped ? p->user_b : p->user_a;
  const void* old_b = p->swapped ? p->user_a : p->user_b;
  CUtensorMap ta = p->tma_a, tb = p->tma_b;
  int32_t is3d = 0;
  if (src_a != old_a) {
    if (p->pack_a) {
      p->pa_src = src_a;
    } else {
      Operand o = p->op_a;
      o.src = src_a;
      const int32_t rc = encode_operand(o, src_a, p->dtype, p->bk, &ta, &is3d);
      if (rc != B2G_OK) return rc;
      if (is3d != p->kp.a_3d) return fail(B2G_ERR_INVALID_ARG, "rebind_layout_changed: create a new plan");
    }
  }
  if (src_b != old_b) {
    if (p->pack_b) {
      p->pb_src = src_b;
    } else {
      Operand o = p->op_b;
      o.src = src_b;
      const int32_t rc = encode_operand(o, src_b, p->dtype, p->bk, &tb, &is3d);
      if (rc != B2G_OK) return rc;
      if (is3d != p->kp.b_3d) return fail(B2G_ERR_INVALID_ARG, "rebind_layout_changed: create a new plan");
    }
  }
  p->tma_a = ta;
  p->tma_b = tb;
  if (p->reduce) p->r_c = C;
  else p->kp.out = C;
  p->user_a = A;
  p->user_b = B;
  p->user_c = C;
  return B2G_OK;
}

int32_t b2g_plan_num_kernels(const b2g_plan* p) {
  if (!p || p->empty) return 0;
  return p->pack_a + p->pack_b + (p->k_zero ? 0 : 1) + p->reduce;
}

int32_t b2g_plan_grid(const b2g_plan* p) { return p ? p->grid : 0; }

int32_t b2g_plan_destroy(b2g_plan* p) {
  delete p;
  return B2G_OK;
}

int32_t b2g_gemm(const b2g_config* cfg, const b2g_problem* prob, const void* A, const void* B, void* C,
                 void* workspace, size_t workspace_bytes, int32_t* status, void* stream) {
  b2g_plan* p = nullptr;
  int32_t rc = b2g_plan_create(cfg, prob, A, B, C, workspace, workspace_bytes, status, &p);
  if (rc != B2G_OK) return rc;
  rc = b2g_plan_launch(p, stream);
  b2g_plan_destroy(p);
  return rc;
}

int32_t b2g_splitk_reduce(const float* ws, void* C, int64_t M, int64_t N, int64_t stride_cm, int64_t stride_cn,
                          int32_t split, int32_t dtype, void* stream) {
  if (M < 0 || N < 0 || split < 0) return fail(B2G_ERR_INVALID_ARG, "negative size");
  if (dtype != B2G_DTYPE_F16 && dtype != B2G_DTYPE_BF16) return fail(B2G_ERR_INVALID_ARG, "bad dtype");
  if (M == 0 || N == 0) return B2G_OK;
  if (!C || (split > 0 && !ws)) return fail(B2G_ERR_INVALID_ARG, "null pointer");
  const int vec = (N % 4 == 0) && stride_cn == 1 && (stride_cm % 4 == 0) &&
                  ((reinterpret_cast<uintptr_t>(C) & 7u) == 0) && ((reinterpret_cast<uintptr_t>(ws) & 15u) == 0);
  const int64_t work = vec ? M * N / 4 : M * N;
  splitk_reduce_kernel<<<grid_for(work, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      ws, C, M, N, stride_cm, stride_cn, split, dtype == B2G_DTYPE_BF16, vec);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(B2G_ERR_CUDA, std::string("launch: ") + cudaGetErrorString(e));
  return B2G_OK;
}

int32_t b2g_gemm_noalloc(const b2g_config* cfg, const b2g_problem* prob, const void* A, const void* B, void* C,
                         int32_t* status, void* stream) {
  Geometry g;
  int32_t rc = make_geometry(cfg, prob, g, A, B, false);
  if (rc != B2G_OK) return rc;
  if (g.streamk)
    return fail(B2G_ERR_UNSUPPORTED,
                "streamk_needs_workspace: stream-K fix-up flags must start zeroed in a caller workspace");
  if (g.a.pack || g.b.pack)
    return fail(B2G_ERR_UNSUPPORTED,
                "operand_needs_staging: the allocation-free entry point reads A and B in place; it needs 16-byte "
                "aligned bases and leading dimensions that are multiples of 8 elements (or unit-stride transposes)");
  if (g.ws_total > kNoAllocScratchBytes) {
    char buf[200];
    snprintf(buf, sizeof buf,
             "split-K partials need %zu bytes; the allocation-free entry point's scratch holds %zu bytes (32 MiB): "
             "lower SPLIT_K or use b2g_plan_create with a workspace",
             g.ws_total, kNoAllocScratchBytes);
    return fail(B2G_ERR_WORKSPACE, buf);
  }
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return fail(B2G_ERR_CUDA, cudaGetErrorString(ce));
  void* scratch = nullptr;
  rc = noalloc_scratch(dev, scratch);
  if (rc != B2G_OK) return rc;
  // Nothing in the scratch needs clearing: each call's GEMM writes every partial element its reduce then reads.
  b2g_plan plan;
  rc = plan_init(&plan, cfg, prob, A, B, C, scratch, kNoAllocScratchBytes, status, false);
  if (rc != B2G_OK) return rc;
  return b2g_plan_launch(&plan, stream);
}

}  // extern "C"
