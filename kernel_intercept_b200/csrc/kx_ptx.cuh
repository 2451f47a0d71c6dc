// kx_ptx.cuh — thin inline-PTX wrappers for the sm_100a features the kx
// kernels use: mbarriers, TMA tiled loads, tcgen05 (TMEM alloc, UMMA issue,
// commit, TMEM loads) and bounded waits.  All waits that depend on another
// agent (TMA engine, tensor core, another warp) are bounded: after
// `timeout_ns` they raise a CTA-wide abort flag and a global error word
// instead of spinning forever.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#define KX_DEV __device__ __forceinline__

namespace kx {

KX_DEV uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

KX_DEV uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

KX_DEV uint32_t lane_id() {
  uint32_t l;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
  return l;
}

// ------------------------------------------------------------- mbarrier ---

KX_DEV void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

KX_DEV void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

KX_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

KX_DEV void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

KX_DEV uint32_t mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P1;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok;
}

// Shared state for bounded waits inside one CTA.
struct WaitCtl {
  volatile int* abort_flag;   // shared memory, 0 = running
  int* err_word;              // global, may be null
  uint64_t timeout_ns;
};

// Wait for the phase with the given parity to complete.  Returns false if the
// CTA is aborting (this wait timed out, or another one did).
KX_DEV bool mbar_wait(uint32_t bar, uint32_t parity, const WaitCtl& w) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = 0;
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 255u) == 0) {
      if (*w.abort_flag) return false;
      uint64_t now = globaltimer();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > w.timeout_ns) {
        *w.abort_flag = 1;
        if (w.err_word) atomicCAS(w.err_word, 0, 3 /* KX_ERR_TIMEOUT */);
        return false;
      }
    }
  }
}

// ------------------------------------------------------------------ TMA ---

KX_DEV void tma_prefetch_desc(const void* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

KX_DEV void tma_load_2d(uint32_t dst, const void* map, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

KX_DEV void tma_load_3d(uint32_t dst, const void* map, uint32_t bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}

// 3-D tile load into this CTA's shared memory whose completion is counted on
// an mbarrier of the peer CTA of a CTA pair (`bar` is a shared::cluster
// address from mapa): the follower of a 2-CTA tile signals the leader's
// stage barrier directly.  No multicast.
KX_DEV void tma_load_3d_pair(uint32_t dst, const void* map, uint32_t bar, int c0, int c1,
                             int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".cta_group::2 [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}

// 4-D tile load of the follower of a CTA pair, counted on the leader's
// barrier (as tma_load_3d_pair).  No multicast.
KX_DEV void tma_load_4d_pair(uint32_t dst, const void* map, uint32_t bar, int c0, int c1, int c2,
                             int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".cta_group::2 [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

KX_DEV void tma_load_4d(uint32_t dst, const void* map, uint32_t bar, int c0, int c1, int c2,
                        int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

// im2col-mode 4-D load {c, w, h, n}: the map's pixelsPerColumn consecutive
// output positions starting at input coordinate (w, h) of image n, walked W,
// then H, then N inside the map's bounding box, each shifted by the filter
// tap offsets (off_w, off_h); channelsPerPixel channels from c per position.
KX_DEV void tma_load_4d_im2col(uint32_t dst, const void* map, uint32_t bar, int c, int w, int h,
                               int n, uint16_t off_w, uint16_t off_h) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], {%7, %8};" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c), "r"(w), "r"(h), "r"(n), "r"(bar),
      "h"(off_w), "h"(off_h)
      : "memory");
}

// im2col-mode 4-D load of the follower of a CTA pair, counted on the
// leader's barrier (as tma_load_3d_pair).  No multicast.
KX_DEV void tma_load_4d_im2col_pair(uint32_t dst, const void* map, uint32_t bar, int c, int w,
                                    int h, int n, uint16_t off_w, uint16_t off_h) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
      ".cta_group::2 [%0], [%1, {%2, %3, %4, %5}], [%6], {%7, %8};" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c), "r"(w), "r"(h), "r"(n), "r"(bar),
      "h"(off_w), "h"(off_h)
      : "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy
// (tensor core operand reads).
KX_DEV void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// TMA stores (shared -> global, bulk async-group completion).  Elements of
// the box outside the tensor are not written.
KX_DEV void tma_store_3d(const void* map, uint32_t src, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

KX_DEV void tma_store_4d(const void* map, uint32_t src, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

KX_DEV void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Wait until at most N committed bulk groups still read shared memory.
template <int N>
KX_DEV void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until every committed bulk group has completed (writes performed).
KX_DEV void bulk_wait_group_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// --------------------------------------------------------------- tcgen05 ---

KX_DEV void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}

KX_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

KX_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

KX_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
KX_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrive on `bar` once every tcgen05.mma issued so far by this thread has
// completed (operands consumed, accumulator written).
KX_DEV void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

KX_DEV void umma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                      uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

KX_DEV void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                     uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// ------------------------------------------------- CTA pairs (cluster 2) --
//
// Two CTAs of a 2-CTA cluster run one tcgen05.mma.cta_group::2 tile: each
// holds half of A's rows and half of B's rows in its own shared memory at the
// same offsets, and half of the accumulator rows in its own TMEM.  Rank 0 (the
// leader) issues the MMAs; remote mbarrier arrivals synchronise the pair.

KX_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
KX_DEV uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

// Arrive on an mbarrier that may live in the peer CTA (address from mapa),
// releasing this thread's prior writes at cluster scope.
KX_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

KX_DEV void st_shared_cluster_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

KX_DEV uint32_t mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P1;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 P1, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok;
}

// mbar_wait with cluster-scope acquire: for barriers the peer CTA arrives on
// (its writes before the arrival are visible after the wait).
KX_DEV bool mbar_wait_cluster(uint32_t bar, uint32_t parity, const WaitCtl& w) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  uint64_t t0 = 0;
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((++spins & 255u) == 0) {
      if (*w.abort_flag) return false;
      uint64_t now = globaltimer();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > w.timeout_ns) {
        *w.abort_flag = 1;
        if (w.err_word) atomicCAS(w.err_word, 0, 3 /* KX_ERR_TIMEOUT */);
        return false;
      }
    }
  }
}

// Every thread of both CTAs: all prior shared-memory work of the pair is done
// and visible (used after barrier init and before TMEM release / exit).
KX_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
                   "memory");
}

KX_DEV void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}

KX_DEV void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

KX_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// Leader only: arrive on `bar` (same offset) in both CTAs of the pair once
// every tcgen05.mma this thread issued has completed.
KX_DEV void tc_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}

KX_DEV void umma_tf32_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

KX_DEV void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns; thread t gets lane (base+t).
KX_DEV void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

KX_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Orders every later use of r after the preceding tcgen05.wait::ld: the
// registers a tcgen05.ld writes are valid only after the wait, and without a
// dependence through them the compiler may schedule their uses earlier.
KX_DEV void tmem_regs_ready(uint32_t (&r)[32]) {
#pragma unroll
  for (int j = 0; j < 32; ++j) asm volatile("" : "+r"(r[j]));
}

// ------------------------------------------------------- UMMA descriptors --
//
// Shared-memory matrix descriptor (sm_100 layout):
//   [0,14)  start address >> 4        [16,30) leading byte offset >> 4
//   [32,46) stride byte offset >> 4   [46,48) version (1 on sm_100)
//   [49,52) base offset               [52]    LBO mode
//   [61,64) layout: 2 = 128-byte swizzle
//
// K-major, 128B swizzle: rows of 128 bytes along K, 8-row (1024 B) atoms;
//   SBO = 1024 (next 8 rows), LBO unused (1).
// MN-major, 128B swizzle: 128-byte chunks along M/N, one row per K index,
//   8 K-rows per 1024 B atom; LBO = byte distance between 128-byte M/N chunks,
//   SBO = 1024 (next 8 K rows).
KX_DEV uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                            uint32_t layout = 2) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}
// Layout 1 (128-byte swizzle of 32-byte atoms) is the only M/N-major layout
// the tensor core accepts for 32-bit (tf32) operands: rows of 128 bytes, one
// per K index, 4-row (512 B) swizzle atoms, so SBO = 512.  TMA writes it with
// CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B.

// Instruction descriptor for kind::tf32 / kind::f16 with an fp32 accumulator.
// fmt: 0 = f16, 1 = bf16, 2 = tf32.  *_mn: operand is M/N-major in smem.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t fmt, bool a_mn, bool b_mn, int M,
                                                  int N) {
  return (1u << 4)                                  // D format = f32
         | (fmt << 7) | (fmt << 10)                 // A, B formats
         | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16)
         | (static_cast<uint32_t>(N >> 3) << 17)   // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);  // M / 16
}

// Round-to-nearest (ties away) fp32 -> tf32, returned as an fp32 value with
// the low 13 mantissa bits cleared.
KX_DEV float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Low part of the 3xTF32 split with a truncated high part:
// x - (x with its low 13 mantissa bits cleared), exact in fp32.  Inf / NaN
// have no low part (their high part carries them).
KX_DEV float tf32_lo(float x) {
  const float t = __uint_as_float(__float_as_uint(x) & 0xffffe000u);
  return isfinite(x) ? x - t : 0.f;
}

}  // namespace kx
