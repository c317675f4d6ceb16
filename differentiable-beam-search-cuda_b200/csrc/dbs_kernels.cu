// sm_100a kernels of the differentiable beam search engine (see dbs_engine.h
// for the decomposition). Arithmetic that decides selection or gradient
// values uses explicitly rounded intrinsics (__fadd_rn, __fmul_rn,
// __fdiv_rn) so nothing is contracted into an FMA: the reference performs
// those operations as separately rounded float ops
// (src/differentiable_beam.cpp:501-506, :1536-1537, :1666, :2108-2111).
#include "dbs_engine.h"

#include <cuda_fp16.h>

#include <cfloat>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <atomic>
#include <mutex>
#include <tuple>
#include <vector>

namespace dbs_dev {

// ---------------------------------------------------------------------------
// Helpers
// ---------------------------------------------------------------------------

// Monotone float -> u32 map; -0 is canonicalised to +0 first so that keys
// compare equal exactly when the floats do (candidate_better uses `!=`).
__device__ __forceinline__ uint32_t ord_f32(float f) {
    uint32_t u = __float_as_uint(__fadd_rn(f, 0.0f));
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float unord_f32(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
    return __uint_as_float(u);
}

// Exact widening of one fp16 / bf16 bit pattern.
__device__ __forceinline__ float widen16(uint32_t h, bool bf16) {
    return bf16 ? __uint_as_float(h << 16) : __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
}

// The 8 values of one 16-byte vector of 16-bit elements, in memory order.
__device__ __forceinline__ void unpack8(const uint4& v, bool bf16, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = widen16(w[i] & 0xFFFFu, bf16);
        f[2 * i + 1] = widen16(w[i] >> 16, bf16);
    }
}

// Log-prob at element index i of the call's input, whatever its width.
__device__ __forceinline__ float lp_at(const DecodeParams& p, int64_t i) {
    return p.x16 ? widen16(__ldg(p.x16 + i), p.x16_bf16 != 0) : __ldg(p.x + i);
}

// Row list entry: larger key = better (lp desc, token asc).
__device__ __forceinline__ uint64_t list_key(float lp, int token) {
    return (static_cast<uint64_t>(ord_f32(lp)) << 32) |
           static_cast<uint64_t>(0xFFFFFFFFu - static_cast<uint32_t>(token));
}
__device__ __forceinline__ float list_lp(uint64_t key) { return unord_f32(static_cast<uint32_t>(key >> 32)); }
__device__ __forceinline__ int list_token(uint64_t key) {
    return static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(key));
}

// Streaming 128-bit load: bypass L1, prefetch the surrounding 256 B into L2.
__device__ __forceinline__ float4 ldg_stream(const float4* p) {
    float4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    return v;
}
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    return v;
}
__device__ __forceinline__ int warp_isum(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// Descending sort of n single-word keys in shared memory with the
// "flip" formulation of bitonic sort: every sorted run has the same
// direction, so out-of-range positions behave as -inf pads that never move and
// n need not be a power of two. Must be called by all threads of the block.
__device__ void block_sort_desc_u64(uint64_t* a, int n) {
    if (n <= 1) { __syncthreads(); return; }
    int n2 = 1;
    while (n2 < n) n2 <<= 1;
    const int half = n2 >> 1;
    for (int size = 2; size <= n2; size <<= 1) {
        const int hs = size >> 1;
        for (int pid = threadIdx.x; pid < half; pid += blockDim.x) {
            const int x = pid & (hs - 1);
            const int blk = (pid - x) << 1;
            const int i = blk + x;
            const int j = blk + size - 1 - x;
            if (j < n) {
                uint64_t ai = a[i], aj = a[j];
                if (ai < aj) { a[i] = aj; a[j] = ai; }
            }
        }
        __syncthreads();
        for (int st = size >> 2; st > 0; st >>= 1) {
            for (int pid = threadIdx.x; pid < half; pid += blockDim.x) {
                const int i = ((pid & ~(st - 1)) << 1) | (pid & (st - 1));
                const int j = i + st;
                if (j < n) {
                    uint64_t ai = a[i], aj = a[j];
                    if (ai < aj) { a[i] = aj; a[j] = ai; }
                }
            }
            __syncthreads();
        }
    }
}

// Same network over two-word keys (hi, lo) compared lexicographically.
__device__ __forceinline__ bool key2_less(uint64_t ah, uint64_t al, uint64_t bh, uint64_t bl) {
    return ah < bh || (ah == bh && al < bl);
}

__device__ void block_sort_desc_u128(uint64_t* hi, uint64_t* lo, int n) {
    if (n <= 1) { __syncthreads(); return; }
    int n2 = 1;
    while (n2 < n) n2 <<= 1;
    const int half = n2 >> 1;
    for (int size = 2; size <= n2; size <<= 1) {
        const int hs = size >> 1;
        for (int pid = threadIdx.x; pid < half; pid += blockDim.x) {
            const int x = pid & (hs - 1);
            const int blk = (pid - x) << 1;
            const int i = blk + x;
            const int j = blk + size - 1 - x;
            if (j < n) {
                uint64_t ih = hi[i], il = lo[i], jh = hi[j], jl = lo[j];
                if (key2_less(ih, il, jh, jl)) { hi[i] = jh; lo[i] = jl; hi[j] = ih; lo[j] = il; }
            }
        }
        __syncthreads();
        for (int st = size >> 2; st > 0; st >>= 1) {
            for (int pid = threadIdx.x; pid < half; pid += blockDim.x) {
                const int i = ((pid & ~(st - 1)) << 1) | (pid & (st - 1));
                const int j = i + st;
                if (j < n) {
                    uint64_t ih = hi[i], il = lo[i], jh = hi[j], jl = lo[j];
                    if (key2_less(ih, il, jh, jl)) { hi[i] = jh; lo[i] = jl; hi[j] = ih; lo[j] = il; }
                }
            }
            __syncthreads();
        }
    }
}

__device__ __forceinline__ int find_example(const int64_t* prefix, int B, int64_t row) {
    int lo = 0, hi = B - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (prefix[mid] <= row) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// Moves the n_top largest (hi, lo) keys of hi/lo[0..m) to the front, sorted
// descending; the rest of the arrays is left in an unspecified order. A
// radix select over the 64-bit hi keys (8 bits per pass, most significant
// first) narrows the keys that can be among the n_top until at most
// `tmp_cap` of them remain; those are gathered into tmp_hi/tmp_lo, sorted and
// copied back. Keys tied on hi beyond that capacity fall back to a full sort.
// Must be called by all threads of the block; ends with a barrier.
// Top n_out keys of nr runs, each sorted descending by (hi, lo) with unique
// keys: run r holds meta_a[r] & 0xFFFF keys at offset meta_a[r] >> 16 of
// (ahi, alo). Rounds of pairwise merges halve the run count; output j of a
// pair comes from a merge-path binary search (how many of the first j come
// from the first run), so a round needs no barrier inside and only the top
// n_out keys of each pair are formed. Rounds ping-pong between (ahi, alo) and
// (bhi, blo); the result is the run at offset 0 of the returned buffer (0 =
// a, 1 = b), *n_res keys. meta_b holds (nr + 1) / 2 words of scratch.
// Called by all threads of the block.
__device__ __noinline__ int block_merge_runs(uint64_t* ahi, uint64_t* alo, uint64_t* bhi, uint64_t* blo,
                                             uint32_t* meta_a, uint32_t* meta_b, int nr, int n_out, int* n_res) {
    __shared__ int sh_total;
    uint64_t *shi = ahi, *slo = alo, *dhi = bhi, *dlo = blo;
    uint32_t *mcur = meta_a, *mnext = meta_b;
    int which = 0;
    while (nr > 1) {
        const int np = (nr + 1) >> 1;
        if (threadIdx.x < 32) {
            // pair lengths (capped at n_out) and their offsets, one warp
            const int lane = threadIdx.x;
            const int per = (np + 31) >> 5;
            const int p0 = lane * per;
            const int p1 = p0 + per < np ? p0 + per : np;
            auto pair_len = [&](int q) {
                int len = static_cast<int>(mcur[2 * q] & 0xFFFFu);
                if (2 * q + 1 < nr) len += static_cast<int>(mcur[2 * q + 1] & 0xFFFFu);
                return len < n_out ? len : n_out;
            };
            int sum = 0;
            for (int q = p0; q < p1; ++q) sum += pair_len(q);
            int incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
                if (lane >= o) incl += v;
            }
            int run = incl - sum;
            for (int q = p0; q < p1; ++q) {
                const int len = pair_len(q);
                mnext[q] = (static_cast<uint32_t>(run) << 16) | static_cast<uint32_t>(len);
                run += len;
            }
            if (lane == 31) sh_total = incl;
        }
        __syncthreads();
        const int total = sh_total;
        for (int g = threadIdx.x; g < total; g += blockDim.x) {
            // the pair holding output g: the last one starting at or before g
            int lo = 0, hi = np - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (static_cast<int>(mnext[mid] >> 16) <= g) lo = mid; else hi = mid - 1;
            }
            const int q = lo;
            const int dst = static_cast<int>(mnext[q] >> 16);
            const int j = g - dst;
            const uint32_t ma = mcur[2 * q];
            const int aoff = static_cast<int>(ma >> 16), a = static_cast<int>(ma & 0xFFFFu);
            int boff = 0, b = 0;
            if (2 * q + 1 < nr) {
                const uint32_t mb = mcur[2 * q + 1];
                boff = static_cast<int>(mb >> 16);
                b = static_cast<int>(mb & 0xFFFFu);
            }
            // i = keys of the first run among the pair's first j outputs
            int l2 = j - b > 0 ? j - b : 0;
            int h2 = j < a ? j : a;
            // x before y: larger high word, or equal high words and larger
            // low word (read only then: high words rarely tie)
            auto before = [&](int x, int y) {
                const uint64_t hx = shi[x], hy = shi[y];
                return hx > hy || (hx == hy && slo[x] > slo[y]);
            };
            while (l2 < h2) {
                const int mid = (l2 + h2) >> 1;
                if (before(aoff + mid, boff + j - 1 - mid)) l2 = mid + 1;
                else h2 = mid;
            }
            const int i = l2;
            bool take_a;
            if (i >= a) take_a = false;
            else if (j - i >= b) take_a = true;
            else take_a = before(aoff + i, boff + j - i);
            const int src = take_a ? aoff + i : boff + j - i;
            dhi[dst + j] = shi[src];
            dlo[dst + j] = slo[src];
        }
        __syncthreads();
        uint64_t* th = shi; shi = dhi; dhi = th;
        uint64_t* tl = slo; slo = dlo; dlo = tl;
        uint32_t* tm = mcur; mcur = mnext; mnext = tm;
        which ^= 1;
        nr = np;
    }
    const int len = nr > 0 ? static_cast<int>(mcur[0] & 0xFFFFu) : 0;
    *n_res = len < n_out ? len : n_out;
    return which;
}

__device__ __noinline__ void block_top_n_u128(uint64_t* hi, uint64_t* lo, int m, int n_top, uint64_t* tmp_hi, uint64_t* tmp_lo,
                                 int tmp_cap) {
    __shared__ int hist[256];
    __shared__ int sh_sel[3];   // chosen digit, keys above the group, keys in the group
    __shared__ int sh_n;
    if (n_top >= m) {
        block_sort_desc_u128(hi, lo, m);
        return;
    }
    // Key 0 marks an empty candidate slot. With at most n_top real keys the
    // answer is all of them, sorted, followed by empty slots.
    if (threadIdx.x == 0) sh_n = 0;
    __syncthreads();
    {
        int c = 0;
        for (int i = threadIdx.x; i < m; i += blockDim.x) c += hi[i] != 0;
        if (c) atomicAdd(&sh_n, c);
    }
    __syncthreads();
    const int real = sh_n;
    __syncthreads();
    if (real <= n_top && real <= tmp_cap) {
        if (threadIdx.x == 0) sh_n = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < m; i += blockDim.x) {
            if (hi[i] != 0) {
                const int pos = atomicAdd(&sh_n, 1);
                tmp_hi[pos] = hi[i];
                tmp_lo[pos] = lo[i];
            }
        }
        __syncthreads();
        block_sort_desc_u128(tmp_hi, tmp_lo, real);
        for (int i = threadIdx.x; i < n_top; i += blockDim.x) {
            hi[i] = i < real ? tmp_hi[i] : 0;
            lo[i] = i < real ? tmp_lo[i] : 0;
        }
        __syncthreads();
        return;
    }
    // aim for a small final sort: at most max(2 n_top, 256) keys
    int target = 2 * n_top < 256 ? 256 : 2 * n_top;
    if (target > tmp_cap) target = tmp_cap;
    uint64_t prefix = 0, mask = 0;
    int need = n_top;
    int above = 0, group = m;
    for (int shift = 56; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < m; i += blockDim.x) {
            const uint64_t k = hi[i];
            if ((k & mask) == prefix) atomicAdd(&hist[static_cast<int>((k >> shift) & 0xFFu)], 1);
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            // digit d* with sum_{d > d*} < need <= sum_{d >= d*}: suffix sums
            // over 8 digits per lane, then across lanes from the top
            const int lane = threadIdx.x;
            int loc[8];
            int tot = 0;
#pragma unroll
            for (int j = 7; j >= 0; --j) {
                loc[j] = hist[lane * 8 + j];
                tot += loc[j];
            }
            int incl = tot;   // inclusive suffix sum over lanes >= lane
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_down_sync(0xFFFFFFFFu, incl, o);
                if (lane + o < 32) incl += v;
            }
            const int excl = incl - tot;   // keys in digits of higher lanes
            if (excl < need && need <= incl) {
                int run = excl;
                for (int j = 7; j >= 0; --j) {
                    if (run + loc[j] >= need) {
                        sh_sel[0] = lane * 8 + j;
                        sh_sel[1] = run;
                        sh_sel[2] = loc[j];
                        break;
                    }
                    run += loc[j];
                }
            }
        }
        __syncthreads();
        const int d = sh_sel[0];
        above += sh_sel[1];
        need -= sh_sel[1];
        group = sh_sel[2];
        prefix |= static_cast<uint64_t>(d) << shift;
        mask |= static_cast<uint64_t>(0xFFu) << shift;
        __syncthreads();   // sh_sel is rewritten by the next pass
        if (above + group <= target) break;
    }
    if (above + group > tmp_cap) {   // massive ties on hi: sort everything
        block_sort_desc_u128(hi, lo, m);
        return;
    }
    // gather every key whose masked prefix is >= the chosen one
    if (threadIdx.x == 0) sh_n = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < m; i += blockDim.x) {
        const uint64_t k = hi[i];
        if ((k & mask) >= prefix) {
            const int pos = atomicAdd(&sh_n, 1);
            tmp_hi[pos] = k;
            tmp_lo[pos] = lo[i];
        }
    }
    __syncthreads();
    const int g = sh_n;
    block_sort_desc_u128(tmp_hi, tmp_lo, g);
    for (int i = threadIdx.x; i < n_top; i += blockDim.x) {
        hi[i] = tmp_hi[i];
        lo[i] = tmp_lo[i];
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------
// 0. Sampled input validation (validate_logprob_tensor,
//    src/differentiable_beam.cpp:385-402): indices 0, s, 2s, ... of the
//    example's tight [T,K,V] tensor, s = count/1000 when count > 1000.
// ---------------------------------------------------------------------------
__global__ void validate_kernel(DecodeParams p) {
    const int e = blockIdx.x;
    const ExampleDesc d = p.desc[e];
    const int64_t V = p.V;
    const int64_t count = static_cast<int64_t>(d.T) * d.K * V;
    const int64_t stride = count > 1000 ? count / 1000 : 1;
    int bad = 0;
    for (int64_t s = threadIdx.x; s * stride < count; s += blockDim.x) {
        const int64_t i = s * stride;
        const int64_t kv = static_cast<int64_t>(d.K) * V;
        const int64_t t = i / kv;
        const int64_t rem = i - t * kv;
        const int64_t k = rem / V;
        const int64_t v = rem - k * V;
        const float x = lp_at(p, d.x_offset + (t * d.k_stride + k) * V + v);
        if (isnan(x) || x == INFINITY) bad = 1;
    }
    bad = __syncthreads_or(bad);
    if (threadIdx.x == 0) p.status[e] = bad ? 1 : 0;
}

// ---------------------------------------------------------------------------
// 1. Row scan: best C entries of every log-prob row.
//
// One warp owns one row at a time; rows are claimed dynamically from a
// global counter, so the load stays balanced to the last row. Each warp
// streams its row body (the 16-byte aligned part) through a private ring of
// kScanStages shared-memory chunks filled by 1-D bulk copies
// (cp.async.bulk, no multicast) that lane 0 issues ahead of the consumption
// point; the prefetch runs on into the next claimed row, so the copy engine
// never waits for the per-row bookkeeping. The unaligned head / tail
// elements are read directly.
//
// Selection is exact and single-pass. An element survives when
// lp >= threshold; everything else only feeds a running max (the bound on what
// was dropped). Finite, statically allowed survivors (banned / EOS before
// min_length) are appended to the warp's buffer with a ballot; a full buffer
// is sorted and cut back to C entries, after which the threshold is "strictly
// above the C-th kept value" (later elements have larger tokens, so an equal
// value can no longer win). The threshold starts at the C-th largest of the
// 32 lane maxima of the first chunk (each lane maximum is a distinct finite,
// allowed element, so at least C candidates reach it), which removes most of
// the first chunk without any guess from other rows.
// ---------------------------------------------------------------------------
constexpr int kScanStages = 4;
constexpr int kScanChunkF4 = 128;       // 2 KB per chunk: 4 float4 per lane
constexpr int kScanWarpsPerCta = 4;
// Lists longer than 32 entries (buffer capacity above 2*32 + 136, plus 128
// for 16-bit rows) compact by radix selection, which needs a 256-bin
// histogram per warp.
__host__ __device__ constexpr int row_scan_hist_ints(int capw, bool k16) {
    return capw - (k16 ? 128 : 0) > 2 * 32 + 136 ? 256 : 0;
}
// Per-warp shared memory: chunk ring | mbarriers | survivor buffer | radix
// histogram | speculation slots (threshold, list length), 128-byte aligned.
__host__ __device__ constexpr size_t row_scan_warp_bytes(int capw, bool k16) {
    return ((static_cast<size_t>(kScanStages) * kScanChunkF4 * 16 + kScanStages * sizeof(uint64_t) +
             static_cast<size_t>(capw) * sizeof(uint64_t) +
             static_cast<size_t>(row_scan_hist_ints(capw, k16)) * sizeof(int) + kSpecSlots * 8) + 127) &
           ~static_cast<size_t>(127);
}

__device__ __forceinline__ void warp_sort_desc_u64(uint64_t* a, int n, int lane) {
    if (n <= 1) { __syncwarp(); return; }
    int n2 = 1;
    while (n2 < n) n2 <<= 1;
    const int half = n2 >> 1;
    for (int size = 2; size <= n2; size <<= 1) {
        const int hs = size >> 1;
        for (int pid = lane; pid < half; pid += 32) {
            const int x = pid & (hs - 1);
            const int blk = (pid - x) << 1;
            const int i = blk + x;
            const int j = blk + size - 1 - x;
            if (j < n) {
                const uint64_t ai = a[i], aj = a[j];
                if (ai < aj) { a[i] = aj; a[j] = ai; }
            }
        }
        __syncwarp();
        for (int st = size >> 2; st > 0; st >>= 1) {
            for (int pid = lane; pid < half; pid += 32) {
                const int i = ((pid & ~(st - 1)) << 1) | (pid & (st - 1));
                const int j = i + st;
                if (j < n) {
                    const uint64_t ai = a[i], aj = a[j];
                    if (ai < aj) { a[i] = aj; a[j] = ai; }
                }
            }
            __syncwarp();
        }
    }
}

// k-th largest (1-based, k <= 32) of one float per lane, broadcast to all lanes.
__device__ __forceinline__ float warp_kth_largest(float v, int k, int lane) {
    // bitonic sort descending across the 32 lanes
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
        for (int st = size >> 1; st > 0; st >>= 1) {
            const float o = __shfl_xor_sync(0xFFFFFFFFu, v, st);
            const bool lower = (lane & st) == 0;
            const bool desc = (lane & size) == 0;
            // keep the larger value in the lower lane of a descending run
            const float hi = fmaxf(v, o), lo = fminf(v, o);
            v = (lower == desc) ? hi : lo;
        }
    }
    return __shfl_sync(0xFFFFFFFFu, v, k - 1);
}

// --- 1-D TMA (cp.async.bulk) + mbarrier helpers ------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Non-multicast bulk copy global -> this CTA's shared memory; completion is
// reported as transaction bytes on `bar`. dst, src and bytes are multiples
// of 16 (the row body is 16-byte aligned by construction).
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}
// Bounded wait: gives up after 2^22 polls (seconds) and reports the timeout
// through the error counter instead of hanging.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned long long* err) {
    for (uint32_t i = 0; i < (1u << 22); ++i)
        if (mbar_try_wait(bar, parity)) return true;
    if (err) atomicExch(err, 1ull);
    return false;
}

// Lists longer than 32 entries: shrink a warp's survivor buffer to the
// entries whose lp is at least the C-th largest lp in it (at least C entries;
// more only when that lp value repeats), keeping token order. The C-th
// largest comes from a radix select over ord(lp) (8 bits per pass, 256-bin
// histogram per warp), so a compaction costs a few passes over the buffer
// instead of a sort. Afterwards only lp strictly above that value can enter
// (a later element with the same lp has a larger token and loses the tie),
// and `evict` holds the largest lp dropped. Called by all lanes of the warp.
__device__ __noinline__ int warp_compact_select(uint64_t* buf, int cnt, int C, int lane, int* hist, float& thr, float& evict) {
    constexpr unsigned FULL = 0xFFFFFFFFu;
    // The keys share their leading bits (similar lp values): start the radix
    // passes at the highest bit where the smallest and largest key differ.
    uint32_t kmin = 0xFFFFFFFFu, kmax = 0;
    for (int i = lane; i < cnt; i += 32) {
        const uint32_t u = static_cast<uint32_t>(buf[i] >> 32);
        kmin = min(kmin, u);
        kmax = max(kmax, u);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        kmin = min(kmin, __shfl_xor_sync(FULL, kmin, o));
        kmax = max(kmax, __shfl_xor_sync(FULL, kmax, o));
    }
    const int top_bit = (kmin == kmax) ? 0 : 31 - __clz(kmin ^ kmax);
    int shift = top_bit >= 8 ? top_bit - 7 : 0;   // digit = bits [shift, shift + 8)
    uint32_t mask = shift + 8 >= 32 ? 0u : ~((1u << (shift + 8)) - 1u);   // bits above the digit
    uint32_t prefix = kmax & mask;   // shared by every key
    int need = C;
    for (;;) {
        for (int i = lane; i < 256; i += 32) hist[i] = 0;
        __syncwarp();
        for (int i = lane; i < cnt; i += 32) {
            const uint32_t u = static_cast<uint32_t>(buf[i] >> 32);
            const bool in = (u & mask) == prefix;
            const int bin = in ? static_cast<int>((u >> shift) & 0xFFu) : -1;
            // lanes with the same bin add once (the leading bits repeat a lot)
            const unsigned act = __activemask();
            const unsigned same = __match_any_sync(act, bin);
            if (in && lane == __ffs(same) - 1) atomicAdd(&hist[bin], __popc(same));
        }
        __syncwarp();
        int loc[8];
        int tot = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            loc[j] = hist[lane * 8 + j];
            tot += loc[j];
        }
        int incl = tot;   // keys in digits of lanes >= this lane
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_down_sync(FULL, incl, o);
            if (lane + o < 32) incl += v;
        }
        const int excl = incl - tot;
        int digit = -1, skipped = 0;
        if (excl < need && need <= incl) {
            int run = excl;
            for (int j = 7; j >= 0; --j) {
                if (run + loc[j] >= need) {
                    digit = lane * 8 + j;
                    skipped = run;
                    break;
                }
                run += loc[j];
            }
        }
        const unsigned owner = __ballot_sync(FULL, digit >= 0);
        const int src = __ffs(owner) - 1;
        digit = __shfl_sync(FULL, digit, src);
        skipped = __shfl_sync(FULL, skipped, src);
        need -= skipped;
        prefix |= static_cast<uint32_t>(digit) << shift;
        mask |= 0xFFu << shift;
        __syncwarp();
        if (shift == 0) break;
        // the last digit may overlap bits already decided: they match the
        // prefix for every key in the group, so the pass stays consistent
        shift = shift >= 8 ? shift - 8 : 0;
    }
    // in-place, order-preserving compaction of the entries with ord(lp) >= prefix
    const unsigned lt = (1u << lane) - 1u;
    float dropped = -INFINITY;
    int w = 0;
    for (int base = 0; base < cnt; base += 32) {
        const int i = base + lane;
        const uint64_t k = i < cnt ? buf[i] : 0;
        const bool keep = i < cnt && static_cast<uint32_t>(k >> 32) >= prefix;
        if (i < cnt && !keep) dropped = fmaxf(dropped, list_lp(k));
        const unsigned b = __ballot_sync(FULL, keep);
        __syncwarp();
        if (keep) buf[w + __popc(b & lt)] = k;
        w += __popc(b);
        __syncwarp();
    }
    evict = fmaxf(evict, warp_max(dropped));
    thr = fmaxf(thr, nextafterf(unord_f32(prefix), INFINITY));
    return w;
}

// Removes banned tokens and the blocked EOS (eos_cut, -1 for none) from a
// warp's survivor buffer, keeping the order; returns the new count. Kept
// out of line: the row scan's hot loop stays as small as without it.
__device__ __noinline__ int warp_drop_disallowed(uint64_t* buf, int cnt, const uint8_t* banned, int eos_cut, int lane) {
    constexpr unsigned FULL = 0xFFFFFFFFu;
    const unsigned lt = (1u << lane) - 1u;
    __syncwarp();
    int w = 0;   // in place: writes stay below the next reads
    for (int base = 0; base < cnt; base += 32) {
        const int i = base + lane;
        const uint64_t key = i < cnt ? buf[i] : 0;
        bool ok = false;
        if (i < cnt) {
            const int v = list_token(key);
            ok = v != eos_cut && !(banned && banned[v]);
        }
        const unsigned b = __ballot_sync(FULL, ok);
        __syncwarp();
        if (ok) buf[w + __popc(b & lt)] = key;
        w += __popc(b);
        __syncwarp();
    }
    return w;
}

struct RowJob {
    const void* row;    // first element of the row (fp32 or 16-bit)
    int64_t r;
    int64_t list_at;  // first list entry of the row
    int C;
    int forced;
    int eos;
    bool eos_blocked;
    bool dead;   // never read: no live parent can extend it
    bool apart;  // scanned by the launch for the step-0 rows
    const uint8_t* banned;
    const uint8_t* allow;   // host filter verdicts of this row, or nullptr
    int h;       // unaligned head elements
    int nv;      // float4 in the aligned body
    int chunks;
};

template <bool k16>
__device__ __forceinline__ float row_lp(const RowJob& j, int i, bool bf16) {
    if constexpr (k16) return widen16(static_cast<const uint16_t*>(j.row)[i], bf16);
    else return static_cast<const float*>(j.row)[i];
}

template <bool k16, bool kFused>
__device__ __forceinline__ RowJob make_job(const DecodeParams& p, int64_t r, int& e) {
    if constexpr (kFused) e = static_cast<int>(r / p.step_major_tk);   // uniform batch: rows jump between examples
    else while (r >= p.row_prefix[e + 1]) ++e;
    const ExampleDesc& d = p.desc[e];
    RowJob j;
    const int64_t lr = r - d.row_begin;
    const int t = static_cast<int>(lr / d.K);
    const int k = static_cast<int>(lr - static_cast<int64_t>(t) * d.K);
    const int64_t elem = d.x_offset + (static_cast<int64_t>(t) * d.k_stride + k) * p.V;
    if constexpr (k16) j.row = p.x16 + elem;
    else j.row = p.x + elem;
    j.r = r;
    // a step's lists: K rows of C entries, then beam 0's extra entries
    j.list_at = d.list_offset + static_cast<int64_t>(t) * (static_cast<int64_t>(d.K) * d.C + d.ext0) +
                static_cast<int64_t>(k) * d.C;
    // the live step-0 row of a short-list decode keeps a long list in the
    // list space of step 0's K rows
    j.C = p.first_rows_only ? min(min(d.N, d.K * d.C), kStep0ListMax) : d.C + (k == 0 ? d.ext0 : 0);
    j.forced = d.forced ? d.forced[t] : -1;
    // A decode starts from beam 0 alone (the other beams score -inf), so the
    // rows of the other beams at step 0 can never yield a candidate; like
    // the reference, which scans live parents only, they are not read.
    j.dead = t == 0 && k > 0;
    j.apart = p.first_row_apart && !p.first_rows_only && t == 0 && k == 0;
    j.eos = d.eos;
    j.eos_blocked = d.eos >= 0 && (t + 1) < d.min_length;
    j.banned = d.banned;
    j.allow = p.row_allow ? p.row_allow + static_cast<int64_t>(k) * p.V : nullptr;
    // head elements up to the first 16-byte boundary, then 16-byte vectors
    constexpr int kShift = k16 ? 1 : 2;   // log2(element bytes)
    const uintptr_t addr = reinterpret_cast<uintptr_t>(j.row);
    int h = static_cast<int>(((16u - (addr & 15u)) & 15u) >> kShift);
    if (h > p.V) h = p.V;
    j.h = h;
    j.nv = (p.V - h) >> (4 - kShift);
    j.chunks = (j.forced >= 0 || j.dead || j.apart) ? 0 : (j.nv + kScanChunkF4 - 1) / kScanChunkF4;
    return j;
}

// Speculative thresholds of long lists left by the warps that last ran out
// of rows in a row-scan launch on this device, (list length << 32) | lp bits
// per slot: a launch's warps start from them instead of from nothing (a row
// whose list a guess cuts short is scanned again, so any value is safe).
__device__ unsigned long long g_spec_seed[kSpecSlots];

__device__ __forceinline__ void scan_row_done(unsigned int* step_done, int idx, int lane) {
    __threadfence();
    __syncwarp();
    if (lane == 0) atomicAdd(step_done + idx, 1u);
}

// The row-scan loop of one warp (per-warp shared memory at smem_raw + warp
// index * row_scan_warp_bytes). With step_done, each finished row (its list,
// count and bound written and fenced) adds one to step_done[e * T + t].
template <bool k16, bool kFused>
__device__ __forceinline__ void row_scan_body(const DecodeParams& p, int capw, int speculate, unsigned char* smem_raw,
                                              unsigned int* step_done) {
    constexpr unsigned FULL = 0xFFFFFFFFu;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // per-warp region: ring | barriers | survivor buffer
    const size_t ring_bytes = static_cast<size_t>(kScanStages) * kScanChunkF4 * 16;
    const int hist_ints = row_scan_hist_ints(capw, k16);
    unsigned char* base = smem_raw + warp * row_scan_warp_bytes(capw, k16);
    float4* ring = reinterpret_cast<float4*>(base);
    uint64_t* full = reinterpret_cast<uint64_t*>(base + ring_bytes);
    uint64_t* buf = full + kScanStages;
    int* hist = reinterpret_cast<int*>(buf + capw);
    float* spec_lp = reinterpret_cast<float*>(hist + hist_ints);   // [kSpecSlots]
    int* spec_len = reinterpret_cast<int*>(spec_lp + kSpecSlots);   // [kSpecSlots], 0 = empty
    unsigned long long* err = p.counters ? p.counters + 3 : nullptr;
    unsigned long long* next_row = p.counters + 2;
    const bool bf16 = p.x16_bf16 != 0;
    const unsigned lt_mask = (1u << lane) - 1u;

    if (lane == 0) {
        for (int s = 0; s < kScanStages; ++s) mbar_init(full + s, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int s = 0; s < kSpecSlots; ++s) {
            const unsigned long long seed = g_spec_seed[s];
            spec_len[s] = static_cast<int>(seed >> 32);
            spec_lp[s] = __uint_as_float(static_cast<uint32_t>(seed));
        }
    }
    __syncwarp();
    // a warp that runs out of rows leaves its thresholds for later launches
    auto leave_seeds = [&]() {
        if (lane == 0)
            for (int s = 0; s < kSpecSlots; ++s)
                if (spec_len[s] > 0)
                    g_spec_seed[s] = (static_cast<unsigned long long>(spec_len[s]) << 32) | __float_as_uint(spec_lp[s]);
    };

    // Claim index -> row (kNoRow once this launch's claims are used up).
    constexpr int64_t kNoRow = INT64_MAX;
    auto claim = [&]() -> int64_t {
        unsigned long long r = 0;
        if (lane == 0) r = atomicAdd(next_row, 1ull);
        r = __shfl_sync(FULL, r, 0);
        if (p.first_rows_only)   // claim i: the first row of example i
            return r < static_cast<unsigned long long>(p.B) ? p.row_prefix[r] : kNoRow;
        if (r >= static_cast<unsigned long long>(p.total_rows)) return kNoRow;
        if constexpr (kFused) {
            // claim order: step, then example, then beam
            const int64_t c = static_cast<int64_t>(r);
            const int64_t t = c / p.step_major_bk;
            const int64_t rem = c - t * p.step_major_bk;
            const int64_t kk = p.step_major_bk / p.B;   // beams per step
            const int64_t b = rem / kk;
            return b * p.step_major_tk + t * kk + (rem - b * kk);
        }
        return static_cast<int64_t>(r);
    };

    // two-row window: `cur` is consumed, `nxt` is being prefetched
    int e_cur = 0, e_nxt = 0;
    int64_t r_cur = claim();
    if (r_cur == kNoRow) return;
    e_cur = find_example(p.row_prefix, p.B, r_cur);
    RowJob cur = make_job<k16, kFused>(p, r_cur, e_cur);
    e_nxt = e_cur;
    RowJob nxt = cur;
    bool have_nxt = false;
    // Issue cursor: the next chunk to copy, the chunks of its row still to
    // copy and the bytes of that row's last chunk; `inxt` once the cursor has
    // moved on to the prefetched row.
    const float4* ip = nullptr;
    int ileft = 0;
    uint32_t ilast = 0;
    bool inxt = false;
    auto cursor_to = [&](const RowJob& jr) {
        ip = reinterpret_cast<const float4*>(static_cast<const char*>(jr.row) +
                                             (static_cast<size_t>(jr.h) << (k16 ? 1 : 2)));
        ileft = jr.chunks;
        ilast = static_cast<uint32_t>(jr.nv - (jr.chunks - 1) * kScanChunkF4) * 16u;
    };
    cursor_to(cur);
    uint32_t n_issued = 0, n_used = 0;

    auto issue_more = [&]() {
        // lane 0 keeps up to kScanStages chunks in flight, crossing into nxt
        while (n_issued < n_used + kScanStages) {
            if (ileft == 0) {
                if (inxt) break;  // at most one row ahead
                // move the issue cursor to the next claimed row
                if (!have_nxt) {
                    const int64_t rn = claim();
                    if (rn == kNoRow) break;
                    nxt = make_job<k16, kFused>(p, rn, e_nxt);
                    have_nxt = true;
                }
                inxt = true;
                cursor_to(nxt);
                continue;
            }
            const uint32_t s = n_issued % kScanStages;
            if (lane == 0) {
                const uint32_t bytes = ileft == 1 ? ilast : kScanChunkF4 * 16u;
                mbar_arrive_expect_tx(full + s, bytes);
                bulk_copy_g2s(ring + s * kScanChunkF4, ip, bytes, full + s);
            }
            ip += kScanChunkF4;
            --ileft;
            ++n_issued;
        }
    };

    // Lists longer than 32 (when each warp scans many rows): the warp starts
    // a row at a speculative threshold, the (C + 6 sqrt(C))-th largest lp of
    // the last row with the same list length C it scanned (the rank of a
    // row's C-th value varies by about sqrt(C) between rows of one
    // distribution). If fewer than C entries reach it the row is scanned
    // again from global memory, so the list stays exact; otherwise far fewer
    // elements take the slow path than with a threshold that starts at
    // -FLT_MAX. (Measured at C = 64 on 256 examples of log_softmax(N(0,1))
    // rows: margins of 3 / 4 / 5 / 6 / 7 / 8 sqrt(C) read 6.4 / 2.4 / 0.8 /
    // 0.15 / 0.01 / 0 % of the rows twice and scan in 21.3 / 18.8 / 17.7 /
    // 17.8 / 17.8 / 28.2 ms.) The guesses are kept per list length in a few
    // slots (the slot that holds C, else an empty one, else one by a hash of
    // C): consecutive rows of a warp come from different examples, whose
    // beam sizes may differ, and beam 0's rows may list more entries; two
    // lengths that shared a slot would evict each other's guess.
    auto spec_slot = [&](int c) {
        for (int s = 0; s < kSpecSlots; ++s)
            if (spec_len[s] == c) return s;
        for (int s = 0; s < kSpecSlots; ++s)
            if (spec_len[s] == 0) return s;
        return static_cast<int>((static_cast<uint32_t>(c) * 2654435761u) >> 30);
    };
    while (true) {
        issue_more();
        const RowJob& j = cur;
        const int C = j.C;
        uint64_t* out = p.lists + j.list_at;
        if (j.apart) {
            // listed by the step-0 launch
        } else if (j.dead) {
            if (lane == 0) {
                p.list_count[j.r] = 0;
                p.list_bound[j.r] = -INFINITY;
            }
        } else if (j.forced >= 0) {
            // Forced step: only the forced token is a candidate of this row.
            if (lane == 0) {
                const float lp = row_lp<k16>(j, j.forced, bf16);
                const bool ok = isfinite(lp) && !(j.banned && j.banned[j.forced]) &&
                                !(j.eos_blocked && j.forced == j.eos) && !(j.allow && !j.allow[j.forced]);
                if (ok) out[0] = list_key(lp, j.forced);
                p.list_count[j.r] = ok ? 1 : 0;
                p.list_bound[j.r] = -INFINITY;
            }
        } else {
            int cnt = 0;
            const int slot = spec_slot(C);
            const float spec = spec_len[slot] == C ? spec_lp[slot] : -FLT_MAX;
            const bool spec_used = speculate && C > 32 && hist_ints && spec > -FLT_MAX;
            float thr = spec_used ? spec : -FLT_MAX;
            float rej = -INFINITY;
            float evict = -INFINITY;
            auto allowed = [&](int v, float lp) {
                return lp != INFINITY && !(j.banned && j.banned[v]) && !(j.eos_blocked && v == j.eos) &&
                       !(j.allow && !j.allow[v]);
            };
            auto consider = [&](bool in, int v, float lp) {
                const bool pass = in && lp >= thr;
                if (in && !pass) rej = fmaxf(rej, lp);
                const bool keep = pass && allowed(v, lp);
                const unsigned b = __ballot_sync(FULL, keep);
                if (keep) buf[cnt + __popc(b & lt_mask)] = list_key(lp, v);
                cnt += __popc(b);
            };
            // Rows without host verdicts append survivors without per-value
            // branches (only +inf is excluded; padding values are -inf, never
            // kept, leaving rej unchanged). Banned tokens and a blocked EOS,
            // which a row has few of, are removed from the survivor buffer
            // afterwards, before each compaction and at the end of the row:
            // a threshold only ever comes from allowed entries.
            const bool plain = !j.allow;
            const bool deferred = j.banned || j.eos_blocked;
            auto drop_disallowed = [&]() {
                if (deferred) cnt = warp_drop_disallowed(buf, cnt, j.banned, j.eos_blocked ? j.eos : -1, lane);
            };
            auto consider_plain = [&](int v, float lp) {
                const bool pass = lp >= thr;
                if (!pass) rej = fmaxf(rej, lp);
                const bool keep = pass && lp != INFINITY;
                const unsigned b = __ballot_sync(FULL, keep);
                if (keep) buf[cnt + __popc(b & lt_mask)] = list_key(lp, v);
                cnt += __popc(b);
            };
            auto compact = [&]() {
                drop_disallowed();
                __syncwarp();
                if (C > 32 && hist_ints) {
                    cnt = warp_compact_select(buf, cnt, C, lane, hist, thr, evict);
                    // room for one more group of appends (128 values, 256
                    // for 16-bit rows) plus the 32-value tail
                    if (cnt <= capw - (k16 ? 256 : 128) - 8 - 32) return;
                    // the C-th lp value repeats too often to free room: cut exactly
                }
                warp_sort_desc_u64(buf, cnt, lane);
                if (cnt > C) {
                    evict = fmaxf(evict, list_lp(buf[C]));
                    thr = fmaxf(thr, nextafterf(list_lp(buf[C - 1]), INFINITY));
                    cnt = C;
                }
                __syncwarp();
            };
            {  // unaligned head, first in token order
                const bool in = lane < j.h;
                const float lp = in ? row_lp<k16>(j, lane, bf16) : -INFINITY;
                consider(in, lane, lp);
            }
            for (int c = 0; c < j.chunks; ++c) {
                const uint32_t s = n_used % kScanStages;
                const uint32_t parity = (n_used / kScanStages) & 1u;
                if (!mbar_wait(full + s, parity, err)) return;
                const float4* st = ring + s * kScanChunkF4;
                float4 q[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) q[u] = st[u * 32 + lane];
                const int nf = j.nv - c * kScanChunkF4;
                if (nf < kScanChunkF4) {
                    // the row's last chunk is partial: the rest of the slot
                    // is stale, read as -inf in the element format
                    const float pad = k16 ? __uint_as_float(bf16 ? 0xFF80FF80u : 0xFC00FC00u) : -INFINITY;
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        if (u * 32 + lane >= nf) q[u] = make_float4(pad, pad, pad, pad);
                }
                if constexpr (!k16) {
                    if (c == 0 && C <= 32) {
                        // threshold bootstrap: C-th largest lane maximum over
                        // finite, allowed elements of the first chunk
                        float mx = -INFINITY;
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            // padding is -inf: not finite, never counted
                            const int v0 = j.h + 4 * (u * 32 + lane);
                            if (isfinite(q[u].x) && allowed(v0 + 0, q[u].x)) mx = fmaxf(mx, q[u].x);
                            if (isfinite(q[u].y) && allowed(v0 + 1, q[u].y)) mx = fmaxf(mx, q[u].y);
                            if (isfinite(q[u].z) && allowed(v0 + 2, q[u].z)) mx = fmaxf(mx, q[u].z);
                            if (isfinite(q[u].w) && allowed(v0 + 3, q[u].w)) mx = fmaxf(mx, q[u].w);
                        }
                        const float kth = warp_kth_largest(mx, C, lane);
                        if (kth > thr) thr = kth;
                    }
                    // the stage is in registers: let lane 0 refill it
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    __syncwarp();
                    ++n_used;
                    issue_more();
                    const int tok0 = j.h + 4 * c * kScanChunkF4;
                    // Fast path: one max and one vote for the lane's 16 values;
                    // survivors are rare once the threshold has settled.
                    float m16 = -INFINITY;
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        m16 = fmaxf(m16, fmaxf(fmaxf(q[u].x, q[u].y), fmaxf(q[u].z, q[u].w)));
                    if (!__any_sync(FULL, m16 >= thr)) {
                        rej = fmaxf(rej, m16);
                    } else {
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            // a 128-value group without a survivor only feeds the bound
                            const float m4 = fmaxf(fmaxf(q[u].x, q[u].y), fmaxf(q[u].z, q[u].w));
                            if (!__any_sync(FULL, m4 >= thr)) {
                                rej = fmaxf(rej, m4);
                                continue;
                            }
                            const int v0 = tok0 + 4 * (u * 32 + lane);
                            if (plain) {
                                consider_plain(v0 + 0, q[u].x);
                                consider_plain(v0 + 1, q[u].y);
                                consider_plain(v0 + 2, q[u].z);
                                consider_plain(v0 + 3, q[u].w);
                            } else {
                                consider(true, v0 + 0, q[u].x);
                                consider(true, v0 + 1, q[u].y);
                                consider(true, v0 + 2, q[u].z);
                                consider(true, v0 + 3, q[u].w);
                            }
                            if (cnt > capw - 128 - 8) compact();
                        }
                    }
                } else {
                    // 16-bit elements: the lane's 4 vectors hold 32 values,
                    // vector w covering tokens tok0 + 8 * (w * 32 + lane) + 0..7
                    const uint4* q16 = reinterpret_cast<const uint4*>(q);
                    float m8[4];
#pragma unroll
                    for (int w = 0; w < 4; ++w) {
                        float f[8];
                        unpack8(q16[w], bf16, f);
                        m8[w] = -INFINITY;
#pragma unroll
                        for (int i = 0; i < 8; ++i) m8[w] = fmaxf(m8[w], f[i]);
                    }
                    if (c == 0 && C <= 32) {
                        float mx = -INFINITY;
#pragma unroll
                        for (int w = 0; w < 4; ++w) {
                            float f[8];
                            unpack8(q16[w], bf16, f);
                            const int v0 = j.h + 8 * (w * 32 + lane);
#pragma unroll
                            for (int i = 0; i < 8; ++i)
                                if (isfinite(f[i]) && allowed(v0 + i, f[i])) mx = fmaxf(mx, f[i]);
                        }
                        const float kth = warp_kth_largest(mx, C, lane);
                        if (kth > thr) thr = kth;
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    __syncwarp();
                    ++n_used;
                    issue_more();
                    const int tok0 = j.h + 8 * c * kScanChunkF4;
                    const float m32 = fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3]));
                    if (!__any_sync(FULL, m32 >= thr)) {
                        rej = fmaxf(rej, m32);
                    } else {
#pragma unroll
                        for (int w = 0; w < 4; ++w) {
                            if (!__any_sync(FULL, m8[w] >= thr)) {
                                rej = fmaxf(rej, m8[w]);
                                continue;
                            }
                            float f[8];
                            unpack8(q16[w], bf16, f);
                            const int v0 = tok0 + 8 * (w * 32 + lane);
#pragma unroll
                            for (int i = 0; i < 8; ++i) {
                                if (plain) consider_plain(v0 + i, f[i]);
                                else consider(true, v0 + i, f[i]);
                            }
                            if (cnt > capw - 256 - 8) compact();
                        }
                    }
                }
            }
            {  // unaligned tail, last in token order
                const int t0 = j.h + (k16 ? 8 : 4) * j.nv;
                const bool in = lane < p.V - t0;
                const float lp = in ? row_lp<k16>(j, t0 + lane, bf16) : -INFINITY;
                consider(in, t0 + lane, lp);
            }
            __syncwarp();
            drop_disallowed();
            const int k_spec = C + static_cast<int>(6.0f * sqrtf(static_cast<float>(C)));
            const bool missed = spec_used && cnt < C;
            if (missed) {
                if (lane == 0 && p.counters) atomicAdd(p.counters, 1ull);   // diagnostics: second passes
                // The speculative threshold dropped part of the best C: scan
                // the row again (global memory, token order). No compaction
                // ran, so the buffer holds every candidate at or above the
                // threshold and each lane's `rej` is the largest element it
                // rejected. Without constraints on the row those 32 maxima
                // are distinct candidates, so the m-th largest of them, for
                // C - cnt <= m <= 32, has at least C candidates at or above
                // it: a safe threshold for the second pass, taken with m up
                // to k_spec - cnt so the next row's threshold can come from it.
                float boot = -FLT_MAX;
                if (C - cnt <= 32 && !j.banned && !j.eos_blocked && !j.allow) {
                    const int m = min(32, k_spec - cnt);
                    const float kth = warp_kth_largest(rej, m, lane);
                    if (kth > boot) boot = kth;   // -inf when fewer than m lanes rejected a finite value
                }
                cnt = 0;
                thr = boot;
                rej = -INFINITY;
                evict = -INFINITY;
                for (int base = 0; base < p.V; base += 128) {
                    const int t0 = base + 4 * lane;
                    float v4[4];
                    bool in4[4];
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        in4[c] = t0 + c < p.V;
                        v4[c] = in4[c] ? row_lp<k16>(j, t0 + c, bf16) : -INFINITY;
                    }
                    const float m4 = fmaxf(fmaxf(v4[0], v4[1]), fmaxf(v4[2], v4[3]));
                    if (!__any_sync(FULL, m4 >= thr)) {
                        rej = fmaxf(rej, m4);
                        continue;
                    }
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        if (plain) consider_plain(t0 + c, v4[c]);
                        else consider(in4[c], t0 + c, v4[c]);
                    }
                    if (cnt > capw - 128 - 8) compact();
                }
                __syncwarp();
                drop_disallowed();
            }
            // long lists: cut to k_spec entries (the next row's speculative
            // threshold comes from there) before the one full sort of the row
            if (C > 32 && hist_ints && cnt > k_spec + 32)
                cnt = warp_compact_select(buf, cnt, k_spec, lane, hist, thr, evict);
            warp_sort_desc_u64(buf, cnt, lane);
            if (C > 32 && hist_ints) {
                float next = spec;
                if (cnt >= k_spec) next = list_lp(buf[k_spec - 1]);
                else if (missed) next = cnt > 0 ? list_lp(buf[cnt - 1]) : -FLT_MAX;   // lower it after a miss
                __syncwarp();
                if (lane == 0) {
                    spec_lp[slot] = next;
                    spec_len[slot] = C;
                }
                __syncwarp();
            }
            const int keep = cnt < C ? cnt : C;
            // beam 0's entries past C go behind the step's K row lists
            const int base_c = p.first_rows_only ? C : p.desc[e_cur].C;
            const int skip = keep > base_c ? (p.desc[e_cur].K - 1) * base_c : 0;
            for (int i = lane; i < keep; i += 32) out[i < base_c ? i : i + skip] = buf[i];
            rej = warp_max(rej);
            if (lane == 0) {
                float b = fmaxf(rej, evict);
                if (cnt > C) b = fmaxf(b, list_lp(buf[C]));
                p.list_count[j.r] = keep;
                p.list_bound[j.r] = b;
            }
            __syncwarp();
        }
        if constexpr (kFused) {
            // step_done[e * T + t] of a uniform batch (row r = e * T * K + t * K + k)
            const int64_t e = j.r / p.step_major_tk;
            const int64_t kk = p.step_major_bk / p.B;
            const int t = static_cast<int>((j.r - e * p.step_major_tk) / kk);
            scan_row_done(step_done, static_cast<int>(e * (p.step_major_tk / kk)) + t, lane);
        }
        // advance to the next claimed row
        if (!inxt) {
            // nothing of the next row was issued yet (nor claimed)
            const int64_t rn = claim();
            if (rn == kNoRow) {
                leave_seeds();
                return;
            }
            nxt = make_job<k16, kFused>(p, rn, e_nxt);
            cursor_to(nxt);
        }
        cur = nxt;
        have_nxt = false;
        inxt = false;
        e_cur = e_nxt;
    }
}

template <bool k16>
__global__ void __launch_bounds__(kScanWarpsPerCta * 32, 4) row_scan_kernel(DecodeParams p, int capw, int speculate) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    row_scan_body<k16, false>(p, capw, speculate, smem_raw, nullptr);
}

// ---------------------------------------------------------------------------
// 2. Step merge: one CTA per example, T sequential steps.
// ---------------------------------------------------------------------------
struct MergeState {
    float* prev_raw;
    float* next_raw;
    int* prev_len;
    int* next_len;
    int* ended;
    int* ended_next;
    int* row_cnt;
    float* row_bound;
    int* unsafe;
    int* blocked_n;   // [K] count of n-gram blocked tokens (constraints only)
};

// Candidate key (hi, lo), larger = better under candidate_better
// (src/differentiable_beam.cpp:291-298): score desc, raw desc, parent asc,
// token asc. Length and from_logprob never decide because (parent, token) is
// unique among a step's candidates (a parent either scans or carries).
__device__ __forceinline__ uint64_t cand_hi(float rank, float raw) {
    return (static_cast<uint64_t>(ord_f32(rank)) << 32) | ord_f32(raw);
}
__device__ __forceinline__ uint64_t cand_lo(int parent, int token) {
    return (static_cast<uint64_t>(0x7FFFFFFFu - static_cast<uint32_t>(parent)) << 32) |
           static_cast<uint64_t>(0x7FFFFFFFu - static_cast<uint32_t>(token));
}
__device__ __forceinline__ int cand_parent(uint64_t lo) {
    return static_cast<int>(0x7FFFFFFFu - static_cast<uint32_t>(lo >> 32));
}
__device__ __forceinline__ int cand_token(uint64_t lo) {
    return static_cast<int>(0x7FFFFFFFu - static_cast<uint32_t>(lo));
}
__device__ __forceinline__ float cand_rank(uint64_t hi) { return unord_f32(static_cast<uint32_t>(hi >> 32)); }
__device__ __forceinline__ float cand_raw(uint64_t hi) { return unord_f32(static_cast<uint32_t>(hi)); }

// Membership in a short list in global memory: eight independent loads per
// round instead of one dependent load per entry.
__device__ __forceinline__ bool in_list(const int32_t* a, int n, int v) {
    int i = 0;
    for (; i + 8 <= n; i += 8) {
        int32_t w[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) w[u] = a[i + u];
        bool hit = false;
#pragma unroll
        for (int u = 0; u < 8; ++u) hit |= w[u] == v;
        if (hit) return true;
    }
    for (; i < n; ++i)
        if (a[i] == v) return true;
    return false;
}

// kRuns: the instance for up to 1024 candidates per step, which merges the
// sorted row runs when no sequence constraint is active (the larger-step
// instance leaves that code out: it costs registers on the selection path).
// Per-beam prefix filters of the step merge (repetition penalty, 1-gram
// blocking): 2^bloom_log2 bits (2048 for up to 32 beams, else 1024), two
// bits per token; a token whose two bits are not both set is not in the
// prefix, and only the others scan it.
__device__ __forceinline__ uint32_t bloom_h1(int v, int lg) { return static_cast<uint32_t>(v) & ((1u << lg) - 1u); }
__device__ __forceinline__ uint32_t bloom_h2(int v, int lg) {
    return (static_cast<uint32_t>(v) * 2654435761u) >> (32 - lg);
}

template <bool kRuns>
__global__ void __launch_bounds__(kMergeThreads, 1) step_merge_kernel(DecodeParams p, int cand_cap,
                                                                   int seq_T, int seq_K, int sel_cap, int bloom_log2,
                                                                   int seq_smem) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int e = blockIdx.x;
    const ExampleDesc d = p.desc[e];
    const int K = d.K, C = d.C, N = d.N, T = d.T, P = d.P;
    const int V = p.V;
    const int tid = threadIdx.x;
    const int NT = blockDim.x;

    uint64_t* chi = reinterpret_cast<uint64_t*>(smem);
    uint64_t* clo = chi + cand_cap;
    float* f_base = reinterpret_cast<float*>(clo + cand_cap);
    MergeState s;
    s.prev_raw = f_base;
    s.next_raw = s.prev_raw + K;
    s.row_bound = s.next_raw + K;
    int* i_base = reinterpret_cast<int*>(s.row_bound + K);
    s.prev_len = i_base;
    s.next_len = s.prev_len + K;
    s.ended = s.next_len + K;
    s.ended_next = s.ended + K;
    s.row_cnt = s.ended_next + K;
    s.unsafe = s.row_cnt + K;
    s.blocked_n = s.unsafe + K;
    // selection scratch after the per-beam arrays (sized by the call's largest K)
    uint64_t* sel_hi = reinterpret_cast<uint64_t*>(
        (reinterpret_cast<uintptr_t>(f_base + 3 * seq_K + 7 * seq_K) + 15) & ~static_cast<uintptr_t>(15));
    uint64_t* sel_lo = sel_hi + sel_cap;
    __shared__ int sh_any_unsafe;
    __shared__ int sh_stage;

    const bool use_rep = p.repetition_penalty > 1.0f;
    const bool use_ngram = p.no_repeat_ngram > 0;
    const bool need_seq = use_rep || use_ngram || p.force_seq;
    // Beam prefixes (with repetition penalty / n-gram constraints / filters):
    // [2][K][seq_T] in global scratch, plus n-gram blocked sets [K][seq_T].
    // per-example region of 3 * seq_K * seq_T (seq_K = largest K of the call)
    int32_t* seq_a = need_seq ? p.seq_scratch + static_cast<int64_t>(e) * 3 * seq_K * seq_T : nullptr;
    int32_t* seq_b = need_seq ? seq_a + static_cast<int64_t>(K) * seq_T : nullptr;
    int32_t* blk = need_seq ? seq_b + static_cast<int64_t>(K) * seq_T : nullptr;
    __shared__ int seq_len_a[1024];
    __shared__ int seq_len_b[1024];
    int* sl_prev = seq_len_a;
    int* sl_next = seq_len_b;

    // beam state: fresh at step 0, else what the previous launch stored
    const int t_first = p.t_begin > 0 ? p.t_begin : 0;
    const int t_stop = p.t_end < T ? p.t_end : T;
    float* state = p.merge_state ? p.merge_state + static_cast<int64_t>(e) * 4 * seq_K : nullptr;
    for (int k = tid; k < K; k += NT) {
        if (t_first > 0 && state) {
            s.prev_raw[k] = state[k];
            s.prev_len[k] = __float_as_int(state[seq_K + k]);
            s.ended[k] = __float_as_int(state[2 * seq_K + k]);
            if (need_seq) sl_prev[k] = __float_as_int(state[3 * seq_K + k]);
        } else {
            s.prev_raw[k] = (k == 0) ? 0.0f : -INFINITY;
            s.prev_len[k] = 0;
            s.ended[k] = 0;
            if (need_seq) sl_prev[k] = 0;
        }
    }
    if (need_seq && (t_first & 1)) {   // the prefix buffers swap once per step
        int32_t* tmp = seq_a; seq_a = seq_b; seq_b = tmp;
    }
    // prefix filters (with the prefixes of an earlier launch, if any)
    const bool use_bloom = need_seq && bloom_log2 > 0;
    const int bl_lg = bloom_log2;
    const int bl_words = use_bloom ? 1 << (bloom_log2 - 5) : 0;
    uint32_t* bloom_a = use_bloom ? reinterpret_cast<uint32_t*>(sel_lo + sel_cap) : nullptr;
    uint32_t* bloom_b = use_bloom ? bloom_a + seq_K * bl_words : nullptr;
    if (use_bloom) {
        for (int i = tid; i < K * bl_words; i += NT) bloom_a[i] = 0;
    }
    // Prefixes and n-gram sets in shared memory when they fit: the launch
    // works on its own copy, loaded from the global scratch when an earlier
    // launch left prefixes there and stored back when a later one continues.
    const bool seq_local = need_seq && seq_smem;
    int32_t* const g_seq = need_seq ? p.seq_scratch + static_cast<int64_t>(e) * 3 * seq_K * seq_T : nullptr;
    if (seq_local) {
        int32_t* sq = reinterpret_cast<int32_t*>(sel_lo + sel_cap) + 2 * seq_K * bl_words;
        __syncthreads();   // prefix lengths of the state loop
        if (t_first > 0) {
            for (int idx = tid; idx < K * seq_T; idx += NT)
                if (idx - (idx / seq_T) * seq_T < sl_prev[idx / seq_T]) sq[idx] = seq_a[idx];
        }
        seq_a = sq;
        seq_b = sq + static_cast<int64_t>(K) * seq_T;
        blk = seq_b + static_cast<int64_t>(K) * seq_T;
    }
    __syncthreads();
    if (use_bloom && t_first > 0) {
        for (int idx = tid; idx < K * seq_T; idx += NT) {
            const int k = idx / seq_T;
            const int i = idx - k * seq_T;
            if (i < sl_prev[k]) {
                const int v = seq_a[static_cast<int64_t>(k) * seq_T + i];
                const uint32_t a = bloom_h1(v, bl_lg), b = bloom_h2(v, bl_lg);
                atomicOr(bloom_a + k * bl_words + (a >> 5), 1u << (a & 31));
                atomicOr(bloom_a + k * bl_words + (b >> 5), 1u << (b & 31));
            }
        }
    }
    __syncthreads();
    // token v in beam k's prefix
    auto in_prefix = [&](int k, int v) {
        if (use_bloom) {
            const uint32_t* bl = bloom_a + k * bl_words;
            const uint32_t a = bloom_h1(v, bl_lg), b = bloom_h2(v, bl_lg);
            if (!((bl[a >> 5] >> (a & 31)) & (bl[b >> 5] >> (b & 31)) & 1u)) return false;
        }
        return in_list(seq_a + static_cast<int64_t>(k) * seq_T, sl_prev[k], v);
    };

    for (int t = t_first; t < t_stop; ++t) {
        const int64_t row0 = d.row_begin + static_cast<int64_t>(t) * K;
        const int forced = d.forced ? d.forced[t] : -1;
        const bool eos_blocked = d.eos >= 0 && (t + 1) < d.min_length;
        const bool ngram_sets = use_ngram && p.no_repeat_ngram >= 2;
        for (int k = tid; k < K; k += NT) {
            s.row_cnt[k] = p.list_count[row0 + k];
            s.row_bound[k] = p.list_bound[row0 + k];
            s.unsafe[k] = 0;
            if (!ngram_sets) s.blocked_n[k] = 0;
        }
        if (ngram_sets) {
            // would_repeat_ngram (src/differentiable_beam.cpp:305-325) as the
            // set of tokens it rejects after each live beam's prefix: one
            // warp per beam, lane i testing the n-gram that starts at i
            const int n = p.no_repeat_ngram;
            const int lane = tid & 31;
            for (int k = tid >> 5; k < K; k += NT >> 5) {
                int cnt = 0;
                const int plen = sl_prev[k];
                if (isfinite(s.prev_raw[k]) && !(d.eos >= 0 && s.ended[k]) && plen + 1 >= n) {
                    const int32_t* pre = seq_a + static_cast<int64_t>(k) * seq_T;
                    int32_t* out = blk + static_cast<int64_t>(k) * seq_T;
                    const int suffix = plen - (n - 1);
                    for (int base = 0; base + n <= plen; base += 32) {
                        const int i = base + lane;
                        bool same = i + n <= plen;
                        for (int q = 0; q < n - 1 && same; ++q) same = pre[i + q] == pre[suffix + q];
                        const unsigned b = __ballot_sync(0xFFFFFFFFu, same);
                        if (same) out[cnt + __popc(b & ((1u << lane) - 1u))] = pre[i + n - 1];
                        cnt += __popc(b);
                    }
                }
                if (lane == 0) s.blocked_n[k] = cnt;
            }
        }
        if (tid == 0) { sh_any_unsafe = 0; sh_stage = 0; }
        __syncthreads();

        // Candidate generation: slot k*C + i holds entry i of row k; an
        // ended parent's carry candidate takes slot k*C. Step 0 of a
        // short-list decode has one live row whose list fills all K*C slots
        // (slot i holds its entry i: the runs of C slots stay sorted).
        const int M = K * C;
        const bool long0 = p.first_row_apart && t == 0;
        for (int idx0 = tid; idx0 < M; idx0 += 4 * NT) {
            // four list loads in flight per thread before any is used
            uint64_t lk[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int idx = idx0 + u * NT;
                lk[u] = 0;
                if (idx < M) {
                    const int k = long0 ? 0 : idx / C;
                    const int i = idx - k * C;
                    if (i < s.row_cnt[k] && isfinite(s.prev_raw[k]) && !(d.eos >= 0 && s.ended[k]))
                        lk[u] = p.lists[d.list_offset + (row0 - d.row_begin + k) * C + i];
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
            const int idx = idx0 + u * NT;
            if (idx >= M) continue;
            const int k = long0 ? 0 : idx / C;
            const int i = idx - k * C;
            uint64_t h = 0, l = 0;
            const float pr = s.prev_raw[k];
            if (isfinite(pr)) {
                if (d.eos >= 0 && s.ended[k]) {
                    if (i == 0) {
                        const int len = s.prev_len[k] < 1 ? 1 : s.prev_len[k];
                        const float rank = __fdiv_rn(pr, p.pen[len]);
                        h = cand_hi(rank, pr);
                        l = cand_lo(k, d.eos);
                    }
                } else if (i < s.row_cnt[k]) {
                    const uint64_t key = lk[u];
                    float lp = list_lp(key);
                    const int v = list_token(key);
                    bool ok = true;
                    if (need_seq) {
                        if (use_ngram) {
                            if (p.no_repeat_ngram == 1) ok = !in_prefix(k, v);
                            else ok = !in_list(blk + static_cast<int64_t>(k) * seq_T, s.blocked_n[k], v);
                        }
                        if (ok && use_rep && in_prefix(k, v))
                            lp = __fsub_rn(lp, p.log_repetition_penalty);
                    }
                    if (ok) {
                        const float raw = __fadd_rn(pr, lp);
                        if (raw != -INFINITY) {
                            const float rank = __fmul_rn(raw, p.inv_pen[s.prev_len[k] + 1]);
                            h = cand_hi(rank, raw);
                            l = cand_lo(k, v);
                        }
                    }
                }
            }
            chi[idx] = h;
            clo[idx] = l;
            }
        }
        __syncthreads();
        bool merged = false;
        if (kRuns && !need_seq && M <= 1024) {   // (the first round then fits the selection buffer)
            // Without per-beam changes to the log-probs each row's candidates
            // come sorted: the list is in (lp desc, token asc) order, and
            // raw = pr + lp and rank = raw * inv only round monotonically.
            // The exception is two lp values rounding to one (rank, raw) with
            // their tokens out of order: such neighbours are swapped (rounds
            // of odd-even transposition restricted to equal high words, so
            // nothing else moves) before the top N is merged from the K
            // sorted runs; a step whose runs stay unsorted sorts.
            uint32_t* meta_a = reinterpret_cast<uint32_t*>(seq_len_a);
            uint32_t* meta_b = reinterpret_cast<uint32_t*>(seq_len_b);
            for (int k = tid; k < K; k += NT) {
                int lo = 0, hi = C;   // empty slots (key 0) only trail a run
                while (lo < hi) {
                    const int mid = (lo + hi) >> 1;
                    if (chi[k * C + mid] != 0) lo = mid + 1; else hi = mid;
                }
                meta_a[k] = (static_cast<uint32_t>(k * C) << 16) | static_cast<uint32_t>(lo);
            }
            int bad = 0;    // neighbours whose high words are out of order (or a gap before a key)
            int ties = 0;   // neighbours with one high word whose tokens are out of order
            for (int idx = tid; idx < M; idx += NT) {
                if (idx % C == C - 1) continue;
                const uint64_t h0 = chi[idx], h1 = chi[idx + 1];
                if (h1 > h0) bad = 1;
                else if (h0 != 0 && h0 == h1 && clo[idx] < clo[idx + 1]) ties = 1;
            }
            bad = __syncthreads_or(bad);
            ties = __syncthreads_or(ties);
            // a group of r equal high words is in order after r rounds; two
            // quiet rounds in a row (one of each parity) mean every group is
            int quiet = 0;
            for (int round = 0; !bad && ties && quiet < 2 && round < 16; ++round) {
                int swapped = 0;
                for (int j = tid; 2 * j + (round & 1) + 1 < M; j += NT) {
                    const int idx = 2 * j + (round & 1);
                    if (idx % C == C - 1) continue;
                    if (chi[idx] != 0 && chi[idx] == chi[idx + 1] && clo[idx] < clo[idx + 1]) {
                        const uint64_t l0 = clo[idx];
                        clo[idx] = clo[idx + 1];
                        clo[idx + 1] = l0;
                        swapped = 1;
                    }
                }
                quiet = __syncthreads_or(swapped) ? 0 : quiet + 1;
            }
            if (ties && quiet < 2) bad = 1;   // still unsorted after 16 rounds: sort the step
            if (!bad) {
                int n_res = 0;
                const int w = block_merge_runs(chi, clo, sel_hi, sel_lo, meta_a, meta_b, K, N, &n_res);
                const int lim = N < M ? N : M;
                for (int i = tid; i < lim; i += NT) {
                    const uint64_t h = i < n_res ? (w ? sel_hi[i] : chi[i]) : 0;
                    const uint64_t l = i < n_res ? (w ? sel_lo[i] : clo[i]) : 0;
                    chi[i] = h;
                    clo[i] = l;
                }
                __syncthreads();
                merged = true;
            }
        }
        if (!merged) {
            if (M > 1024) block_top_n_u128(chi, clo, M, N, sel_hi, sel_lo, sel_cap);
            else block_sort_desc_u128(chi, clo, M);
        }

        // Exactness proof per truncated row: every entry the scan dropped has
        // lp <= bound, so its candidate is at most U = (rank(bound),
        // raw(bound)); if the current N-th candidate G beats U, no dropped
        // entry can enter the top-N.
        for (int k = tid; k < K; k += NT) {
            const float pr = s.prev_raw[k];
            if (!isfinite(pr) || (d.eos >= 0 && s.ended[k])) continue;
            const float bnd = s.row_bound[k];
            if (!(bnd > -INFINITY)) continue;  // nothing dropped
            const float raw_u = __fadd_rn(pr, bnd);
            if (raw_u == -INFINITY) continue;   // dropped entries can never be selected
            const float rank_u = __fmul_rn(raw_u, p.inv_pen[s.prev_len[k] + 1]);
            bool safe = false;
            if (N - 1 < M && chi[N - 1] != 0) {
                const uint64_t uh = cand_hi(rank_u, raw_u);
                const uint64_t gh = chi[N - 1];
                safe = gh > uh || (gh == uh && cand_parent(clo[N - 1]) < k);
            }
            if (!safe) {
                s.unsafe[k] = 1;
                atomicOr(&sh_any_unsafe, 1);
            }
        }
        __syncthreads();

        if (sh_any_unsafe) {
            // Rescan the unproven rows from HBM and merge in every dropped
            // candidate that beats the current N-th (rare path).
            const int stage_room = cand_cap - N;
            for (int k = 0; k < K; ++k) {
                if (!s.unsafe[k]) continue;
                if (tid == 0 && p.counters) atomicAdd(p.counters + 1, 1ull);
                const float pr = s.prev_raw[k];
                const float inv = p.inv_pen[s.prev_len[k] + 1];
                const int64_t row = d.x_offset + (static_cast<int64_t>(t) * d.k_stride + k) * V;
                const int cnt = s.row_cnt[k];
                const uint64_t last = p.lists[d.list_offset + (row0 - d.row_begin + k) * C + (cnt - 1)];
                const float m_lp = list_lp(last);
                const int m_tok = list_token(last);
                // lp floor for the N-th candidate G = (gh, .): a value f whose
                // candidate, formed with the same roundings, has a high word
                // below G's; rounding is monotone, so no lp <= f can beat G (a
                // penalised lp is lower still). -inf when that cannot be shown.
                auto floor_of = [&](uint64_t gh) {
                    float floor_lp = -INFINITY;
                    if (gh != 0) {
                        const float rg = cand_rank(gh);
                        float f = __fsub_rn(__fdiv_rn(rg, inv), pr);
                        f = __fsub_rn(f, (fabsf(f) + fabsf(pr) + 1.0f) * 1e-3f);
                        const float rawf = __fadd_rn(pr, f);
                        const float rankf = __fmul_rn(rawf, inv);
                        if (isfinite(f) && isfinite(rawf) && isfinite(rankf) && cand_hi(rankf, rawf) < gh) floor_lp = f;
                    }
                    return floor_lp;
                };
                // The candidate of token v when the scan dropped it and it
                // beats G = (gh, gl); false otherwise.
                auto dropped_winner = [&](int v, float lp, float floor_lp, uint64_t gh, uint64_t gl, uint64_t& h,
                                          uint64_t& l) -> bool {
                    if (lp <= floor_lp) return false;   // (NaN falls through to the check below)
                    if (forced >= 0 && v != forced) return false;
                    if (d.banned && d.banned[v]) return false;
                    if (eos_blocked && v == d.eos) return false;
                    if (p.row_allow && !p.row_allow[static_cast<int64_t>(k) * V + v]) return false;
                    if (!isfinite(lp)) return false;
                    const float lpc = __fadd_rn(lp, 0.0f);
                    if (lpc > m_lp || (lpc == m_lp && v <= m_tok)) return false;  // already listed
                    if (need_seq) {
                        if (use_ngram) {
                            const bool bl = (p.no_repeat_ngram == 1)
                                                ? in_prefix(k, v)
                                                : in_list(blk + static_cast<int64_t>(k) * seq_T, s.blocked_n[k], v);
                            if (bl) return false;
                        }
                        if (use_rep && in_prefix(k, v)) lp = __fsub_rn(lp, p.log_repetition_penalty);
                    }
                    const float raw = __fadd_rn(pr, lp);
                    if (raw == -INFINITY) return false;
                    const float rank = __fmul_rn(raw, inv);
                    h = cand_hi(rank, raw);
                    l = cand_lo(k, v);
                    return key2_less(gh, gl, h, l);
                };
                // Merges the `staged` keys behind the top N into it; leaves
                // the stage empty. Called by all threads.
                auto merge_staged = [&](int staged) {
                    if (staged <= 64) {
                        // A few staged keys (the usual case): the final
                        // position of a key of the sorted top N is its
                        // index plus the staged keys above it; that of a
                        // staged key is the top-N keys above it (binary
                        // search) plus the staged keys above it. Keys are
                        // unique, so the positions below N are distinct.
                        for (int i = tid; i < N + staged; i += NT) {
                            const uint64_t h = chi[i], l = clo[i];
                            int pos = 0;
                            if (i < N) {
                                pos = i;
                                for (int q = N; q < N + staged; ++q) pos += key2_less(h, l, chi[q], clo[q]) ? 1 : 0;
                            } else {
                                int lo = 0, hi = N;   // top-N keys above (h, l)
                                while (lo < hi) {
                                    const int mid = (lo + hi) >> 1;
                                    if (key2_less(h, l, chi[mid], clo[mid])) lo = mid + 1; else hi = mid;
                                }
                                pos = lo;
                                for (int q = N; q < N + staged; ++q) pos += key2_less(h, l, chi[q], clo[q]) ? 1 : 0;
                            }
                            if (pos < N) {
                                sel_hi[pos] = h;
                                sel_lo[pos] = l;
                            }
                        }
                        __syncthreads();
                        for (int i = tid; i < N; i += NT) {
                            chi[i] = sel_hi[i];
                            clo[i] = sel_lo[i];
                        }
                    } else if (N + staged > 1024) {
                        block_top_n_u128(chi, clo, N + staged, N, sel_hi, sel_lo, sel_cap);
                    } else {
                        block_sort_desc_u128(chi, clo, N + staged);
                    }
                    for (int i = N + tid; i < N + staged; i += NT) { chi[i] = 0; clo[i] = 0; }
                    __syncthreads();
                    if (tid == 0) sh_stage = 0;
                    __syncthreads();
                };

                // One sweep against the G of the row's start: 16 loads per
                // thread in flight, no barrier until the row ends, winners
                // staged through a shared counter and merged once. If more
                // winners than the staging room holds turn up (G far from
                // settled), the row is swept again in batches that merge as
                // they go.
                {
                    const uint64_t gh = (N - 1 < M) ? chi[N - 1] : 0;
                    const uint64_t gl = (N - 1 < M) ? clo[N - 1] : 0;
                    const float floor_lp = floor_of(gh);
                    for (int base = 0; base < V; base += 16 * NT) {
                        float lv[16];
#pragma unroll
                        for (int r = 0; r < 16; ++r) {
                            const int v = base + r * NT + tid;
                            lv[r] = v < V ? lp_at(p, row + v) : -INFINITY;
                        }
#pragma unroll
                        for (int r = 0; r < 16; ++r) {
                            const int v = base + r * NT + tid;
                            uint64_t h, l;
                            if (v < V && dropped_winner(v, lv[r], floor_lp, gh, gl, h, l)) {
                                const int pos = atomicAdd(&sh_stage, 1);
                                if (pos < stage_room) {
                                    chi[N + pos] = h;
                                    clo[N + pos] = l;
                                }
                            }
                        }
                    }
                }
                __syncthreads();
                const int swept = sh_stage;
                __syncthreads();
                if (swept <= stage_room) {
                    if (swept > 0) merge_staged(swept);
                    continue;
                }
                if (tid == 0) sh_stage = 0;
                __syncthreads();
                // Sub-batches of 4 values per thread (4 NT <= 2048 <= the
                // room); four sub-batches (16 loads per thread) are in flight
                // before the first is used. After each sub-batch the staged
                // candidates are merged if the room could overflow, and G is
                // re-read (it only improves).
                const int sub = 4 * NT;
                for (int base = 0; base < V; base += 4 * sub) {
                    float lv[16];
#pragma unroll
                    for (int r = 0; r < 16; ++r) {
                        const int v = base + (r >> 2) * sub + (r & 3) * NT + tid;
                        lv[r] = v < V ? lp_at(p, row + v) : -INFINITY;
                    }
#pragma unroll
                    for (int sb = 0; sb < 4; ++sb) {
                        const int sbase = base + sb * sub;
                        if (sbase >= V) break;
                        const uint64_t gh = (N - 1 < M) ? chi[N - 1] : 0;
                        const uint64_t gl = (N - 1 < M) ? clo[N - 1] : 0;
                        const float floor_lp = floor_of(gh);
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int v = sbase + u * NT + tid;
                            uint64_t h, l;
                            if (v < V && dropped_winner(v, lv[sb * 4 + u], floor_lp, gh, gl, h, l)) {
                                const int pos = atomicAdd(&sh_stage, 1);
                                chi[N + pos] = h;
                                clo[N + pos] = l;
                            }
                        }
                        __syncthreads();
                        const int staged = sh_stage;
                        __syncthreads();   // every thread holds the count before the next sub-batch stages
                        const bool last_sub = sbase + sub >= V;
                        if (staged > 0 && (last_sub || staged > stage_room - sub)) merge_staged(staged);
                    }
                }
            }
        }

        // Outputs of step t and beam state update.
        const bool want_pool = p.pool_scores != nullptr;
        for (int j = tid; j < N; j += NT) {
            const uint64_t h = (j < M) ? chi[j] : 0;
            const uint64_t l = (j < M) ? clo[j] : 0;
            int parent = -1, token = -1, len = 0, flp = 0;
            float rank = -INFINITY, raw = -INFINITY;
            if (h != 0) {
                parent = cand_parent(l);
                token = cand_token(l);
                rank = cand_rank(h);
                raw = cand_raw(h);
                const bool carry = d.eos >= 0 && s.ended[parent];
                len = carry ? (s.prev_len[parent] < 1 ? 1 : s.prev_len[parent]) : s.prev_len[parent] + 1;
                flp = carry ? 0 : 1;
            }
            if (want_pool && j < P) {
                const int64_t o = d.pool_offset + static_cast<int64_t>(t) * d.pool_t_stride + j;
                p.pool_parents[o] = parent;
                p.pool_tokens[o] = token;
                p.pool_lengths[o] = len;
                p.pool_raw_scores[o] = raw;
                p.pool_scores[o] = rank;
                if (p.pool_from_logprob) p.pool_from_logprob[o] = static_cast<uint8_t>(flp);
            }
            if (j < K) {
                const int64_t o = d.sel_offset + static_cast<int64_t>(t) * d.sel_t_stride + j;
                p.parents[o] = parent;
                p.tokens[o] = token;
                p.lengths[o] = len;
                if (p.raw_scores) p.raw_scores[o] = raw;
                if (p.scores) p.scores[o] = rank;
                p.from_logprob[o] = static_cast<uint8_t>(flp);
                s.next_raw[j] = raw;
                s.next_len[j] = len;
                s.ended_next[j] = (parent >= 0) ? ((s.ended[parent] != 0) || (d.eos >= 0 && token == d.eos)) : 0;
            }
        }
        __syncthreads();
        if (need_seq) {
            // prefix[j] = prefix[parent_j] ++ token_j (when from a log-prob)
            for (int j = tid; j < K; j += NT) {
                const uint64_t l = (j < M) ? clo[j] : 0;
                const uint64_t h = (j < M) ? chi[j] : 0;
                int len = 0;
                if (h != 0) {
                    const int parent = cand_parent(l);
                    len = sl_prev[parent];
                    const bool carry = d.eos >= 0 && s.ended[parent];
                    if (!carry) len += 1;
                }
                sl_next[j] = len;
            }
            for (int idx = tid; idx < K * seq_T; idx += NT) {
                const int j = idx / seq_T;
                const int i = idx - j * seq_T;
                const uint64_t h = (j < M) ? chi[j] : 0;
                if (h == 0) continue;
                const uint64_t l = clo[j];
                const int parent = cand_parent(l);
                const int plen = sl_prev[parent];
                if (i < plen) seq_b[static_cast<int64_t>(j) * seq_T + i] = seq_a[static_cast<int64_t>(parent) * seq_T + i];
                else if (i == plen && !(d.eos >= 0 && s.ended[parent]))
                    seq_b[static_cast<int64_t>(j) * seq_T + i] = cand_token(l);
            }
        }
        if (use_bloom) {
            // filter[j] = filter[parent_j] + token_j (when from a log-prob)
            for (int idx = tid; idx < K * bl_words; idx += NT) {
                const int j = idx / bl_words;
                const int w = idx - j * bl_words;
                const uint64_t h = (j < M) ? chi[j] : 0;
                uint32_t bits = 0;
                if (h != 0) {
                    const uint64_t l = clo[j];
                    const int parent = cand_parent(l);
                    bits = bloom_a[parent * bl_words + w];
                    if (!(d.eos >= 0 && s.ended[parent])) {
                        const int v = cand_token(l);
                        const uint32_t a = bloom_h1(v, bl_lg), b = bloom_h2(v, bl_lg);
                        if (static_cast<int>(a >> 5) == w) bits |= 1u << (a & 31);
                        if (static_cast<int>(b >> 5) == w) bits |= 1u << (b & 31);
                    }
                }
                bloom_b[idx] = bits;
            }
        }
        __syncthreads();
        for (int k = tid; k < K; k += NT) {
            s.prev_raw[k] = s.next_raw[k];
            s.prev_len[k] = s.next_len[k];
            s.ended[k] = s.ended_next[k];
        }
        if (need_seq) {
            int32_t* tmp = seq_a; seq_a = seq_b; seq_b = tmp;
            int* tl = sl_prev; sl_prev = sl_next; sl_next = tl;
            uint32_t* tb = bloom_a; bloom_a = bloom_b; bloom_b = tb;
        }
        __syncthreads();
    }
    if (t_stop < T) {   // more steps follow in a later launch: keep the state
        if (seq_local) {
            // the later launch starts from the buffer its step's parity names
            int32_t* g_cur = g_seq + ((t_stop & 1) ? static_cast<int64_t>(K) * seq_T : 0);
            for (int idx = tid; idx < K * seq_T; idx += NT)
                if (idx - (idx / seq_T) * seq_T < sl_prev[idx / seq_T]) g_cur[idx] = seq_a[idx];
        }
        if (state) {
            for (int k = tid; k < K; k += NT) {
                state[k] = s.prev_raw[k];
                state[seq_K + k] = __int_as_float(s.prev_len[k]);
                state[2 * seq_K + k] = __int_as_float(s.ended[k]);
                state[3 * seq_K + k] = __int_as_float(need_seq ? sl_prev[k] : 0);
            }
        }
        return;
    }
    // Finalisation (src/differentiable_beam.cpp:1661-1667): a division, not
    // a multiply by the reciprocal.
    for (int k = tid; k < K; k += NT) {
        const int len = s.prev_len[k] < 1 ? 1 : s.prev_len[k];
        const int64_t o = d.final_offset + k;
        if (p.final_raw_scores) p.final_raw_scores[o] = s.prev_raw[k];
        if (p.final_scores) p.final_scores[o] = __fdiv_rn(s.prev_raw[k], p.pen[len]);
    }
}

// ---------------------------------------------------------------------------
// 2c. Compact selection merge (no repetition penalty / n-gram blocking /
//     prefix-keeping, at most 8 * NT candidates per step, pools up to NT).
//
// One CTA of NT threads per example walks its steps. Every thread owns
// kLmPer candidate slots of a step (slot idx = tid + u * NT: entry idx % C
// of row idx / C) and holds their 64-bit (rank, raw) keys and tokens in
// registers, so a step needs no shared-memory copy of its K row lists. A
// radix select over the 128-bit candidate keys (rank, raw, then parent and
// token; 8 bits per pass from the highest bit where the keys differ)
// narrows the keys that can be among the top N to at most NT; those are
// gathered and ranked by counting, and the first N are the step's pool (the
// same order as the reference's candidate_better,
// src/differentiable_beam.cpp:291-298). The exactness proof and the
// rescans of truncated rows follow the selection merge.
// ---------------------------------------------------------------------------

// Shared memory of list_merge_body: selection keys and their rank words, the
// histogram and ten per-beam arrays.
__host__ __device__ constexpr size_t list_merge_smem(int nt, int sel_cap, int max_K) {
    return static_cast<size_t>(sel_cap) * (2 * sizeof(uint64_t) + sizeof(uint32_t)) + 256 * sizeof(int) +
           static_cast<size_t>(max_K) * 10 * sizeof(int) + 0 * nt;
}
// Selection buffer: a power of two with room for the top N plus a staging
// area of at least 256 and of at least one value per thread (rescans).
__host__ __device__ constexpr int list_merge_sel_cap(int max_N, int nt) {
    int c = 1;
    while (c < max_N + (nt > 256 ? nt : 256) || c < 2 * max_N) c <<= 1;
    return c;
}

// Descending bitonic sort of n2 (a power of two) two-word keys, (0, 0) pads
// last. Called by all threads of the block; ends with a barrier.
template <int NT>
__device__ __forceinline__ void lm_sort(uint64_t* hi, uint64_t* lo, int n2) {
    const int half = n2 >> 1;
    for (int size = 2; size <= n2; size <<= 1) {
        for (int st = size >> 1; st > 0; st >>= 1) {
            for (int pid = threadIdx.x; pid < half; pid += NT) {
                const int i = ((pid & ~(st - 1)) << 1) | (pid & (st - 1));
                const int j = i + st;
                const bool desc = (i & size) == 0;
                const uint64_t ih = hi[i], jh = hi[j];
                const uint64_t il = lo[i], jl = lo[j];
                const bool i_less = key2_less(ih, il, jh, jl);
                if (i_less == desc) { hi[i] = jh; lo[i] = jl; hi[j] = ih; lo[j] = il; }
            }
            __syncthreads();
        }
    }
}

// Prefetch block of one example in list_merge_body: a flag (set when the
// next step's lists are on their way), then room for pf_cap list entries and
// the next step's K counts and K bounds. 16-byte copies that bypass L1
// (cp.async.cg), so that lines of steps the scan has not listed yet are
// never cached on the SM.
__host__ __device__ constexpr size_t merge_prefetch_bytes(int pf_cap, int max_K) {
    return 16 + static_cast<size_t>(pf_cap) * sizeof(uint64_t) +
           ((static_cast<size_t>(max_K) * 2 * sizeof(int) + 15) & ~static_cast<size_t>(15));
}
__host__ __device__ constexpr size_t align16(size_t n) { return (n + 15) & ~static_cast<size_t>(15); }
__device__ __forceinline__ void cp_async_16_cg(void* smem_dst, const void* gsrc) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit_all() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Bounded wait of a merge CTA for the K rows of step t of example e
// (step_done[e * T + t] == K, counted by the row-scan warps of the same
// launch after their lists are written). Returns false, after setting the
// timeout counter, if the rows do not arrive within about two seconds.
// Called by all threads of the block.
__device__ __forceinline__ bool wait_step_rows(const DecodeParams& p, const unsigned int* step_done, int idx,
                                               unsigned int want) {
    __shared__ int sh_ok;
    if (threadIdx.x == 0) {
        int ok = 1;
        const long long t0 = clock64();
        for (;;) {
            unsigned int v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(step_done + idx) : "memory");
            if (v >= want) break;
            if (clock64() - t0 > (4ll << 30)) {
                ok = 0;
                if (p.counters) atomicExch(p.counters + 3, 1ull);
                break;
            }
            __nanosleep(200);
        }
        sh_ok = ok;
    }
    __syncthreads();
    const bool ok = sh_ok != 0;
    __threadfence();
    __syncthreads();   // sh_ok is read by every thread before it can change
    return ok;
}

// Steps [t_first, t_stop) of example e. state (global, [4][seq_K] for this
// example) carries the beams between calls: loaded when t_first > 0,
// stored when steps remain. With step_done the CTA waits for each step's
// rows (the fused decode); lists, counts and bounds are read around L1.
template <int NT, int PER>
__device__ __forceinline__ bool list_merge_body(const DecodeParams& p, int e, int t_first, int t_stop, float* state,
                                                int seq_K, int sel_cap, unsigned char* smem,
                                                const unsigned int* step_done, float* beams = nullptr,
                                                bool fresh = true, unsigned char* pfb = nullptr,
                                                int pf_cap = 0) {
    constexpr int NW = NT / 32;
    constexpr unsigned FULL = 0xFFFFFFFFu;
    constexpr int kLmPer = PER;
    const ExampleDesc d = p.desc[e];
    const int K = d.K, C = d.C, N = d.N, T = d.T, P = d.P;
    const int V = p.V;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    uint64_t* sh = reinterpret_cast<uint64_t*>(smem);   // [sel_cap] selection / sort keys (high words)
    uint64_t* sl = sh + sel_cap;                         // [sel_cap] low words
    uint32_t* sr = reinterpret_cast<uint32_t*>(sl + sel_cap);   // [sel_cap] rank words of the gathered keys
    int* hist = reinterpret_cast<int*>(sr + sel_cap);    // [256]
    float* prev_raw = reinterpret_cast<float*>(hist + 256);
    float* next_raw = prev_raw + seq_K;
    int* prev_len = reinterpret_cast<int*>(prev_raw + 4 * seq_K);
    int* ended = prev_len + 2 * seq_K;
    if (beams) {   // the example's beams kept in the caller's shared memory between calls
        prev_raw = beams;
        prev_len = reinterpret_cast<int*>(beams + seq_K);
        ended = reinterpret_cast<int*>(beams + 2 * seq_K);
    }
    float* row_bound = next_raw + seq_K;
    float* row_inv = row_bound + seq_K;
    int* next_len = reinterpret_cast<int*>(row_inv + 2 * seq_K);
    int* ended_next = next_len + 2 * seq_K;
    int* row_cnt = ended_next + seq_K;
    int* unsafe = row_cnt + seq_K;
    __shared__ int sh_n;
    __shared__ int sh_g;   // gather counter of the step
    __shared__ int sh_any;
    __shared__ int sh_over;
    __shared__ int sh_sel[3];
    __shared__ unsigned long long sh_mm[2 * NW];
    const bool use_eos = d.eos >= 0;
    if (t_stop > T) t_stop = T;
    __syncthreads();   // the block's previous call is done with the shared arrays
    for (int k = tid; k < K; k += NT) {
        if (t_first > 0 && state && !beams) {
            prev_raw[k] = state[k];
            prev_len[k] = __float_as_int(state[seq_K + k]);
            ended[k] = __float_as_int(state[2 * seq_K + k]);
        } else if (t_first == 0) {
            prev_raw[k] = (k == 0) ? 0.0f : -INFINITY;
            prev_len[k] = 0;
            ended[k] = 0;
        }
    }
    int sort_n2 = 1;
    while (sort_n2 < sel_cap) sort_n2 <<= 1;   // sel_cap is a power of two
    // A step's slots: K rows of C entries (slot k * C + i: entry i of row k),
    // then beam 0's entries C .. C + ext0 - 1 (slot K * C + i - C); at step
    // 0 of a decode with the first row apart, entry i of row 0 (slot i).
    const int KC = K * C;
    const int ext0 = d.ext0;
    // the selection buffer past the top N is the rescans' staging area and
    // is kept zero from here on (the sorts read it; every step leaves it so)
    if (fresh)
        for (int i = tid; i < sort_n2; i += NT) { sh[i] = 0; sl[i] = 0; }
    // the 1 / penalty table in shared memory, so that a step's set-up reads
    // no global memory once its lists are prefetched (published by the step
    // loop's first barrier; every call of a block shares one table)
    constexpr int kInvCache = 512;
    __shared__ float sh_inv[kInvCache];
    const bool inv_cached = p.Lmax + 1 <= kInvCache;
    if (fresh && inv_cached)
        for (int i = tid; i <= p.Lmax; i += NT) sh_inv[i] = p.inv_pen[i];

    for (int t = t_first; t < t_stop; ++t) {
        const int64_t row0 = d.row_begin + static_cast<int64_t>(t) * K;
        const uint64_t* step_lists = p.lists + d.list_offset + static_cast<int64_t>(t) * (KC + ext0);
        const int forced = d.forced ? d.forced[t] : -1;
        const bool eos_blocked = use_eos && (t + 1) < d.min_length;
        // lists, counts and bounds prefetched during the example's previous
        // step (flag 1: entries only, 2: counts and bounds too)
        int* pf_flag = reinterpret_cast<int*>(pfb);
        uint64_t* pf_e = pfb ? reinterpret_cast<uint64_t*>(pfb + 16) : nullptr;
        int* pf_cnt = pfb ? reinterpret_cast<int*>(pf_e + pf_cap) : nullptr;
        float* pf_bnd = pfb ? reinterpret_cast<float*>(pf_cnt + K) : nullptr;
        const int pf_have = pfb ? *pf_flag : 0;   // (read before thread 0 rewrites it below)
        cp_async_wait_all();   // (this thread's copies of any prefetch)
        __syncthreads();   // the previous step's state update and the prefetched lists are visible
        if (step_done && !pf_have && !wait_step_rows(p, step_done, e * T + t, static_cast<unsigned int>(K)))
            return false;
        const bool long0 = p.first_row_apart && t == 0;
        const int M = long0 ? KC : KC + ext0;
        auto slot_row = [&](int idx) { return long0 || idx >= KC ? 0 : idx / C; };
        auto slot_entry = [&](int idx, int k) { return long0 ? idx : (idx >= KC ? C + (idx - KC) : idx - k * C); };
        // The step's list entries (its M slots of the lists) are loaded
        // together with the counts and bounds, one round trip (or read from
        // the prefetch); entries past a row's count are dropped after the
        // barrier.
        uint64_t raw_e[kLmPer];
#pragma unroll
        for (int u = 0; u < kLmPer; ++u) {
            const int idx = tid + u * NT;
            raw_e[u] = idx >= M ? 0ull
                                : (pf_have ? pf_e[idx]
                                           : __ldcg(reinterpret_cast<const unsigned long long*>(step_lists) + idx));
        }
        for (int k = tid; k < K; k += NT) {
            row_cnt[k] = pf_have == 2 ? pf_cnt[k] : __ldcg(p.list_count + row0 + k);
            row_bound[k] = pf_have == 2 ? pf_bnd[k] : __ldcg(p.list_bound + row0 + k);
            row_inv[k] = inv_cached ? sh_inv[prev_len[k] + 1] : p.inv_pen[prev_len[k] + 1];
            unsafe[k] = 0;
            next_raw[k] = INFINITY;   // the lp and token of the row's last listed entry (rescans)
            next_len[k] = -1;
        }
        if (tid == 0) { sh_n = 0; sh_g = 0; sh_any = 0; }
        for (int i = tid; i < 256; i += NT) hist[i] = 0;   // the first radix pass
        const int MN = KC + ext0;   // the next step's slots
        const uint64_t* next_lists = step_lists + MN;
        if (pfb && tid == 0) {
            // prefetch the next step's lists while this step runs, when they
            // are listed (always, without step_done) and fit 16-byte copies
            // (the next step of this example comes in this call, or, with the
            // beams kept by the caller, in its next call)
            int ok = t + 1 < (beams ? T : t_stop) && MN <= pf_cap && (MN & 1) == 0 &&
                     (reinterpret_cast<uintptr_t>(next_lists) & 15u) == 0;
            if (ok && step_done) {
                unsigned int v;
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];"
                             : "=r"(v)
                             : "l"(step_done + e * T + t + 1)
                             : "memory");
                ok = v >= static_cast<unsigned int>(K);
            }
            if (ok && (K & 3) == 0 && (reinterpret_cast<uintptr_t>(p.list_count + row0 + K) & 15u) == 0 &&
                (reinterpret_cast<uintptr_t>(p.list_bound + row0 + K) & 15u) == 0)
                ok = 2;
            *pf_flag = ok;
        }
        __syncthreads();
        if (pfb) {
            const int pf_next = *pf_flag;
            if (pf_next) {
                for (int c = tid; c < (MN >> 1); c += NT) cp_async_16_cg(pf_e + 2 * c, next_lists + 2 * c);
                if (pf_next == 2)
                    for (int c = tid; c < (K >> 2); c += NT) {
                        cp_async_16_cg(pf_cnt + 4 * c, p.list_count + row0 + K + 4 * c);
                        cp_async_16_cg(pf_bnd + 4 * c, p.list_bound + row0 + K + 4 * c);
                    }
                cp_async_commit_all();
            }
        }

        // candidate keys of this thread's slots
        uint64_t ch[kLmPer];
        int ctok[kLmPer];
        {
#pragma unroll
            for (int u = 0; u < kLmPer; ++u) {
                const int idx = tid + u * NT;
                if (idx < M) {
                    const int k = slot_row(idx);
                    const int i = slot_entry(idx, k);
                    if (i == row_cnt[k] - 1) {
                        next_raw[k] = list_lp(raw_e[u]);
                        next_len[k] = list_token(raw_e[u]);
                    }
                    if (!(i < row_cnt[k] && isfinite(prev_raw[k]) && !(use_eos && ended[k]))) raw_e[u] = 0;
                }
            }
#pragma unroll
            for (int u = 0; u < kLmPer; ++u) {
                const int idx = tid + u * NT;
                uint64_t h = 0;
                int tok = -1;
                if (idx < M) {
                    const int k = slot_row(idx);
                    const int i = slot_entry(idx, k);
                    const float pr = prev_raw[k];
                    if (isfinite(pr)) {
                        if (use_eos && ended[k]) {
                            if (i == 0) {   // the ended parent's carry candidate
                                const int len = prev_len[k] < 1 ? 1 : prev_len[k];
                                h = cand_hi(__fdiv_rn(pr, p.pen[len]), pr);
                                tok = d.eos;
                            }
                        } else if (raw_e[u] != 0) {
                            const float raw = __fadd_rn(pr, list_lp(raw_e[u]));
                            if (raw != -INFINITY) {
                                h = cand_hi(__fmul_rn(raw, row_inv[k]), raw);
                                tok = list_token(raw_e[u]);
                            }
                        }
                    }
                }
                ch[u] = h;
                ctok[u] = tok;
            }
        }
        auto cand_lo_of = [&](int u) -> uint64_t {
            return cand_lo(slot_row(tid + u * NT), ctok[u]);
        };

        // Radix select: the masked prefix (ph, pl) that the top-N keys reach
        uint64_t ph = 0, pl = 0, mh = 0, ml = 0;   // prefix and mask over (hi, lo)
        // the gathered keys are ranked by counting (g x g comparisons), one
        // per thread at the end, so at most NT of them; fewer when the
        // radix passes can get there
        const int gather_cap = NT < sel_cap ? NT : sel_cap;
        const int gather_goal = N + 128 < gather_cap ? N + 128 : gather_cap;
        int need = N;
        int total = 0;
        {
            // real candidates and the range of their high words
            unsigned long long mn = ~0ull, mx = 0ull;
            int c = 0;
#pragma unroll
            for (int u = 0; u < kLmPer; ++u) {
                if (ch[u]) {
                    ++c;
                    mn = min(mn, static_cast<unsigned long long>(ch[u]));
                    mx = max(mx, static_cast<unsigned long long>(ch[u]));
                }
            }
            c = warp_isum(c);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                mn = min(mn, __shfl_xor_sync(FULL, mn, o));
                mx = max(mx, __shfl_xor_sync(FULL, mx, o));
            }
            if (lane == 0) {
                atomicAdd(&sh_n, c);
                sh_mm[2 * wid] = mn;
                sh_mm[2 * wid + 1] = mx;
            }
            __syncthreads();
            total = sh_n;
            mn = ~0ull;
            mx = 0ull;
            for (int w = 0; w < NW; ++w) {
                mn = min(mn, sh_mm[2 * w]);
                mx = max(mx, sh_mm[2 * w + 1]);
            }
            __syncthreads();
            if (total > N) {
                // start at the highest bit where the high words differ; the
                // bits above it are shared by every real candidate
                int bit = (mn == mx) ? 0 : 63 - __clzll(static_cast<long long>(mn ^ mx));
                int shift = bit >= 7 ? bit - 7 : 0;   // digit = bits [shift, shift + 8) of the 128-bit key
                bool in_lo = false;
                if (mn == mx) {   // every high word equal: decide on the low words
                    mh = ~0ull;
                    ph = mx;
                    in_lo = true;
                    shift = 56;
                } else {
                    mh = (shift + 8 >= 64) ? 0ull : ~((1ull << (shift + 8)) - 1ull);
                    ph = mx & mh;
                }
                for (bool first = true;; first = false) {
                    if (!first) {
                        for (int i = tid; i < 256; i += NT) hist[i] = 0;
                        __syncthreads();
                    }
                    int* wh = hist;
#pragma unroll
                    for (int u = 0; u < kLmPer; ++u) {
                        int bin = -1;
                        if (ch[u] && (ch[u] & mh) == ph) {
                            if (!in_lo) {
                                bin = static_cast<int>((ch[u] >> shift) & 0xFFu);
                            } else {
                                const uint64_t l = cand_lo_of(u);
                                if ((l & ml) == pl) bin = static_cast<int>((l >> shift) & 0xFFu);
                            }
                        }
                        const unsigned same = __match_any_sync(FULL, bin);
                        if (bin >= 0 && lane == __ffs(same) - 1) atomicAdd(wh + bin, __popc(same));
                    }
                    __syncthreads();
                    if (wid == 0) {
                        // digit d* with sum_{d > d*} < need <= sum_{d >= d*}
                        int loc[8];
                        int tot = 0;
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            loc[j] = hist[lane * 8 + j];
                            tot += loc[j];
                        }
                        int incl = tot;
#pragma unroll
                        for (int o = 1; o < 32; o <<= 1) {
                            const int v = __shfl_down_sync(FULL, incl, o);
                            if (lane + o < 32) incl += v;
                        }
                        const int excl = incl - tot;
                        if (excl < need && need <= incl) {
                            int run = excl;
                            for (int j = 7; j >= 0; --j) {
                                if (run + loc[j] >= need) {
                                    sh_sel[0] = lane * 8 + j;
                                    sh_sel[1] = run;
                                    sh_sel[2] = loc[j];
                                    break;
                                }
                                run += loc[j];
                            }
                        }
                    }
                    __syncthreads();
                    const int digit = sh_sel[0];
                    const int above = sh_sel[1];
                    const int group = sh_sel[2];
                    __syncthreads();   // sh_sel is rewritten by the next pass
                    if (!in_lo) {
                        ph |= static_cast<uint64_t>(digit) << shift;
                        mh |= 0xFFull << shift;
                    } else {
                        pl |= static_cast<uint64_t>(digit) << shift;
                        ml |= 0xFFull << shift;
                    }
                    need -= above;
                    // keys above the group plus the group are few enough to rank
                    if ((N - need) + group <= gather_goal) break;
                    if (shift == 0) {
                        if (in_lo) break;   // (unreachable: low words are unique)
                        in_lo = true;
                        shift = 56;
                    } else {
                        shift = shift >= 8 ? shift - 8 : 0;
                    }
                }
            }
        }
        // The taken candidates: every one whose masked key reaches the prefix.
        bool tk[kLmPer];
#pragma unroll
        for (int u = 0; u < kLmPer; ++u) {
            const uint64_t h = ch[u];
            bool take = false;
            if (h) {
                take = total <= N || (h & mh) > ph;
                if (!take && (h & mh) == ph) {
                    const uint64_t l = cand_lo_of(u);
                    take = ml == 0 || (l & ml) >= pl;
                }
            }
            tk[u] = take;
        }
        // Gather them (one shared atomic per warp) with their rank words,
        // and clear the counts of the ranking.
        int* rank_cnt = reinterpret_cast<int*>(sh + NT);   // [NT]: greater | equal << 16 (sel_cap >= 2 NT)
        for (int i = tid; i < NT; i += NT) rank_cnt[i] = 0;
        if (tid == 0) sh_n = 0;   // the count of tied keys below (the radix total is read)
        {
            unsigned bal[kLmPer];
            int wtot = 0;
#pragma unroll
            for (int u = 0; u < kLmPer; ++u) {
                bal[u] = __ballot_sync(FULL, tk[u]);
                wtot += __popc(bal[u]);
            }
            int base = 0;
            if (lane == 0 && wtot) base = atomicAdd(&sh_g, wtot);
            base = __shfl_sync(FULL, base, 0);
#pragma unroll
            for (int u = 0; u < kLmPer; ++u) {
                if ((bal[u] >> lane) & 1u) {
                    const int pos = base + __popc(bal[u] & ((1u << lane) - 1u));
                    sh[pos] = ch[u];
                    sl[pos] = cand_lo_of(u);
                    sr[pos] = static_cast<uint32_t>(ch[u] >> 32);
                }
                base += __popc(bal[u]);
            }
        }
        __syncthreads();
        {
            // Rank of each gathered key = the gathered keys above it (keys
            // are unique). The g x g comparisons of rank words are cut into
            // work items of (key, 64 words) spread over all threads, four
            // words per broadcast load, counting the greater and the equal
            // words without branches; the items' counts add up in shared
            // memory. A key whose rank word is shared by another (rare)
            // compares the full keys of those. The first N keys move to
            // their slots.
            const int g = sh_g;
            constexpr int kChunk = 64;
            const int parts = (g + kChunk - 1) / kChunk;
            const uint4* sr4 = reinterpret_cast<const uint4*>(sr);
            for (int item = tid; item < parts * g; item += NT) {
                const int part = item / g;
                const int i = item - part * g;
                const uint32_t r = sr[i];
                const int j1 = min(g, (part + 1) * kChunk);
                int gt = 0, eq = 0;
                int j = part * kChunk;
                for (; j + 4 <= j1; j += 4) {
                    const uint4 w = sr4[j >> 2];
                    gt += (w.x > r ? 1 : 0) + (w.y > r ? 1 : 0) + (w.z > r ? 1 : 0) + (w.w > r ? 1 : 0);
                    eq += (w.x == r ? 1 : 0) + (w.y == r ? 1 : 0) + (w.z == r ? 1 : 0) + (w.w == r ? 1 : 0);
                }
                for (; j < j1; ++j) {
                    gt += sr[j] > r ? 1 : 0;
                    eq += sr[j] == r ? 1 : 0;
                }
                atomicAdd(rank_cnt + i, gt | (eq << 16));
            }
            __syncthreads();
            // keys whose rank word another key shares: one warp each counts
            // the keys with that word above it
            constexpr int kTieCap = 64;
            __shared__ int sh_tie[kTieCap];
            if (tid < g && (rank_cnt[tid] >> 16) > 1) {
                const int q = atomicAdd(&sh_n, 1);
                if (q < kTieCap) {
                    sh_tie[q] = tid;
                } else {
                    const uint32_t r = sr[tid];
                    int add = 0;
                    for (int j = 0; j < g; ++j)
                        if (sr[j] == r) add += key2_less(sh[tid], sl[tid], sh[j], sl[j]) ? 1 : 0;
                    atomicAdd(rank_cnt + tid, add);
                }
            }
            __syncthreads();
            const int ties = sh_n < kTieCap ? sh_n : kTieCap;
            for (int q = wid; q < ties; q += NW) {
                const int i = sh_tie[q];
                const uint32_t r = sr[i];
                const uint64_t ih = sh[i], il = sl[i];
                int add = 0;
                for (int j = lane; j < g; j += 32)
                    if (sr[j] == r) add += key2_less(ih, il, sh[j], sl[j]) ? 1 : 0;
                add = warp_isum(add);
                if (lane == 0) atomicAdd(rank_cnt + i, add);
            }
            __syncthreads();
            uint64_t kh = 0, kl = 0;
            int rank = 0;
            if (tid < g) {
                kh = sh[tid];
                kl = sl[tid];
                rank = rank_cnt[tid] & 0xFFFF;
            }
            if (tid == 0) sh_n = 0;
            __syncthreads();
            // the buffer beyond the first N keys is the rescans' staging
            // area, kept zero
            if (tid < g && rank < N) {
                sh[rank] = kh;
                sl[rank] = kl;
            }
            for (int i = (g < N ? g : N) + tid; i < 2 * NT; i += NT) {
                sh[i] = 0;
                sl[i] = 0;
            }
            __syncthreads();
        }

        // Exactness proof per truncated row (as in the selection merge): a
        // dropped entry can beat the N-th key G only if the row's bound U does.
        for (int k = tid; k < K; k += NT) {
            const float pr = prev_raw[k];
            if (!isfinite(pr) || (use_eos && ended[k])) continue;
            const float bnd = row_bound[k];
            if (!(bnd > -INFINITY)) continue;
            const float raw_u = __fadd_rn(pr, bnd);
            if (raw_u == -INFINITY) continue;
            const float rank_u = __fmul_rn(raw_u, row_inv[k]);
            bool safe = false;
            if (sh[N - 1] != 0) {
                const uint64_t uh = cand_hi(rank_u, raw_u);
                const uint64_t gh = sh[N - 1];
                safe = gh > uh || (gh == uh && cand_parent(sl[N - 1]) < k);
            }
            if (!safe) {
                unsafe[k] = 1;
                atomicOr(&sh_any, 1);
            }
        }
        __syncthreads();
        if (sh_any) {
            // Rescan each unproven row from HBM: every candidate the scan
            // dropped that beats the current N-th key G is staged behind the
            // top N and merged in by one sort; a row with more winners than
            // the staging room is swept again against the improved G.
            const int room = sel_cap - N;
            for (int k = 0; k < K; ++k) {
                if (!unsafe[k]) continue;
                if (tid == 0 && p.counters) atomicAdd(p.counters + 1, 1ull);
                const float pr = prev_raw[k];
                const float inv = row_inv[k];
                const int64_t row = d.x_offset + (static_cast<int64_t>(t) * d.k_stride + k) * V;
                // the row's last listed entry (INFINITY / -1 for an empty list)
                const float m_lp = next_raw[k];
                const int m_tok = next_len[k];
                // The candidate of token v if the scan dropped it and it beats
                // G = (gh, gl); 0 otherwise.
                auto winner = [&](int v, float lp, float floor_lp, uint64_t gh, uint64_t gl, uint64_t& l) -> uint64_t {
                    if (!(lp > floor_lp)) return 0;
                    if (forced >= 0 && v != forced) return 0;
                    if (d.banned && d.banned[v]) return 0;
                    if (eos_blocked && v == d.eos) return 0;
                    if (p.row_allow && !p.row_allow[static_cast<int64_t>(k) * V + v]) return 0;
                    if (!isfinite(lp)) return 0;
                    const float lpc = __fadd_rn(lp, 0.0f);
                    if (lpc > m_lp || (lpc == m_lp && v <= m_tok)) return 0;   // listed
                    const float raw = __fadd_rn(pr, lp);
                    if (raw == -INFINITY) return 0;
                    const uint64_t h = cand_hi(__fmul_rn(raw, inv), raw);
                    l = cand_lo(k, v);
                    return key2_less(gh, gl, h, l) ? h : 0;
                };
                // lp floor for G: no lp at or below it forms a candidate above G
                auto floor_of = [&](uint64_t gh) {
                    float floor_lp = -INFINITY;
                    if (gh != 0) {
                        const float rg = cand_rank(gh);
                        float f = __fsub_rn(__fdiv_rn(rg, inv), pr);
                        f = __fsub_rn(f, (fabsf(f) + fabsf(pr) + 1.0f) * 1e-3f);
                        const float rawf = __fadd_rn(pr, f);
                        const float rankf = __fmul_rn(rawf, inv);
                        if (isfinite(f) && isfinite(rawf) && isfinite(rankf) && cand_hi(rankf, rawf) < gh) floor_lp = f;
                    }
                    return floor_lp;
                };
                auto merge_stage = [&](int staged) {   // top N of (top N + staged); called by all threads
                    if (staged <= 128 && N + staged <= 2 * NT) {
                        // the new position of a top-N key is its index plus the
                        // staged keys above it; that of a staged key is the
                        // top-N keys above it (binary search) plus the staged
                        // keys above it
                        uint64_t kh[2], kl[2];
                        int pos[2];
#pragma unroll
                        for (int r = 0; r < 2; ++r) {
                            const int i = tid + r * NT;
                            pos[r] = N;
                            kh[r] = 0;
                            kl[r] = 0;
                            if (i < N + staged) {
                                kh[r] = sh[i];
                                kl[r] = sl[i];
                                int ps = 0;
                                if (i < N) {
                                    ps = i;
                                } else {
                                    int lo = 0, hi = N;
                                    while (lo < hi) {
                                        const int mid = (lo + hi) >> 1;
                                        if (key2_less(kh[r], kl[r], sh[mid], sl[mid])) lo = mid + 1; else hi = mid;
                                    }
                                    ps = lo;
                                }
                                for (int q = N; q < N + staged; ++q) ps += key2_less(kh[r], kl[r], sh[q], sl[q]) ? 1 : 0;
                                pos[r] = ps;
                            }
                        }
                        __syncthreads();
#pragma unroll
                        for (int r = 0; r < 2; ++r) {
                            if (pos[r] < N && kh[r] != 0) {
                                sh[pos[r]] = kh[r];
                                sl[pos[r]] = kl[r];
                            }
                        }
                        __syncthreads();
                        for (int i = N + tid; i < N + staged; i += NT) { sh[i] = 0; sl[i] = 0; }
                        __syncthreads();
                        return;
                    }
                    int n2 = 2;
                    while (n2 < N + staged) n2 <<= 1;
                    lm_sort<NT>(sh, sl, n2);
                    for (int i = N + tid; i < n2; i += NT) { sh[i] = 0; sl[i] = 0; }
                    __syncthreads();
                };
                // The row's values in token order, by all threads: fp32 rows
                // take the scalar head up to a 16-byte boundary and the tail by
                // plain loads and the body as float4 vectors; 16-bit rows take
                // element loads. fn1(v, lp) gets one value, fn4(q, v0) the
                // vector of tokens v0 .. v0 + 3.
                auto sweep_row = [&](auto&& fn1, auto&& fn4) {
                    if (p.x16) {
                        for (int base = 0; base < V; base += 16 * NT) {
                            float lv[16];
#pragma unroll
                            for (int r = 0; r < 16; ++r) {
                                const int v = base + r * NT + tid;
                                lv[r] = v < V ? lp_at(p, row + v) : -INFINITY;
                            }
#pragma unroll
                            for (int r = 0; r < 16; ++r) {
                                const int v = base + r * NT + tid;
                                if (v < V) fn1(v, lv[r]);
                            }
                        }
                        return;
                    }
                    const float* rp = p.x + row;
                    const int head = min(V, static_cast<int>(((16u - (reinterpret_cast<uintptr_t>(rp) & 15u)) & 15u) >> 2));
                    if (tid < head) fn1(tid, rp[tid]);
                    const float4* body = reinterpret_cast<const float4*>(rp + head);
                    const int nv = (V - head) >> 2;
                    for (int base = 0; base < nv; base += 4 * NT) {   // four vectors per thread in flight
                        float4 q[4];
#pragma unroll
                        for (int r = 0; r < 4; ++r) {
                            const int i = base + r * NT + tid;
                            q[r] = i < nv ? __ldg(body + i) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
                        }
#pragma unroll
                        for (int r = 0; r < 4; ++r) {
                            const int i = base + r * NT + tid;
                            if (i < nv) fn4(q[r], head + 4 * i);
                        }
                    }
                    const int t0 = head + 4 * nv;
                    if (t0 + tid < V) fn1(t0 + tid, rp[t0 + tid]);
                };
                // While the step has fewer than N candidates (G empty: step 0 of
                // a decode whose one live row has a short list), every entry of
                // the row would win; only entries at or above the row's N-th
                // largest allowed log-prob can be among the top N. A radix
                // select over the row (8 bits per pass from the top) narrows a
                // prefix of ord(lp) until the values at or above it fit the
                // staging room, and the floor is put just below the prefix.
                float nth_floor = -INFINITY;
                bool over = false;
                // the sweep, and once more above the row's N-th largest allowed
                // value if it stages more winners than the room
                for (int attempt = 0; attempt < 2; ++attempt) {
                    if (sh[N - 1] == 0 || attempt == 1) {
                        uint32_t prefix = 0, mask = 0;
                        int need_r = N;
                        bool enough = true;
                        for (int shift = 24;; shift -= 8) {
                            for (int i = tid; i < 256; i += NT) hist[i] = 0;
                            __syncthreads();
                            auto count = [&](int v, float lp) {
                                int bin = -1;
                                if (isfinite(lp) && !(forced >= 0 && v != forced) && !(d.banned && d.banned[v]) &&
                                    !(eos_blocked && v == d.eos) &&
                                    !(p.row_allow && !p.row_allow[static_cast<int64_t>(k) * V + v])) {
                                    const uint32_t u = ord_f32(lp);
                                    if ((u & mask) == prefix) bin = static_cast<int>((u >> shift) & 0xFFu);
                                }
                                const unsigned act = __activemask();
                                const unsigned same = __match_any_sync(act, bin);
                                if (bin >= 0 && lane == __ffs(same) - 1) atomicAdd(hist + bin, __popc(same));
                            };
                            sweep_row(count, [&](const float4 q, int v0) {
                                count(v0, q.x);
                                count(v0 + 1, q.y);
                                count(v0 + 2, q.z);
                                count(v0 + 3, q.w);
                            });
                            __syncthreads();
                            if (wid == 0) {
                                int loc[8];
                                int tot = 0;
#pragma unroll
                                for (int j = 0; j < 8; ++j) {
                                    loc[j] = hist[lane * 8 + j];
                                    tot += loc[j];
                                }
                                int incl = tot;
#pragma unroll
                                for (int o = 1; o < 32; o <<= 1) {
                                    const int v = __shfl_down_sync(FULL, incl, o);
                                    if (lane + o < 32) incl += v;
                                }
                                const int excl = incl - tot;
                                if (lane == 0 && incl < need_r) sh_sel[0] = -1;   // fewer than N allowed entries
                                if (excl < need_r && need_r <= incl) {
                                    int run = excl;
                                    for (int j = 7; j >= 0; --j) {
                                        if (run + loc[j] >= need_r) {
                                            sh_sel[0] = lane * 8 + j;
                                            sh_sel[1] = run;
                                            sh_sel[2] = loc[j];
                                            break;
                                        }
                                        run += loc[j];
                                    }
                                }
                            }
                            __syncthreads();
                            const int digit = sh_sel[0];
                            const int above = sh_sel[1];
                            const int group = sh_sel[2];
                            __syncthreads();
                            if (digit < 0) { enough = false; break; }
                            prefix |= static_cast<uint32_t>(digit) << shift;
                            mask |= 0xFFu << shift;
                            need_r -= above;
                            // the values at or above the prefix: (N - need_r) + group
                            if (shift == 0 || (N - need_r) + group <= room) break;
                        }
                        if (enough) {
                            const float edge = unord_f32(prefix);   // the least value with the prefix
                            nth_floor = isfinite(edge) ? nextafterf(edge, -INFINITY) : -INFINITY;
                        }
                    }
                    // one sweep against the G of the row's start, no barrier inside
                    {
                        const uint64_t gh = sh[N - 1], gl = sl[N - 1];
                        const float floor_lp = gh == 0 ? nth_floor : fmaxf(floor_of(gh), nth_floor);
                        if (tid == 0) { sh_n = 0; sh_over = 0; }
                        __syncthreads();
                        auto stage = [&](int v, float lp) {
                            uint64_t l = 0;
                            const uint64_t h = winner(v, lp, floor_lp, gh, gl, l);
                            if (!h) return;
                            const int pos = atomicAdd(&sh_n, 1);
                            if (pos < room) {
                                sh[N + pos] = h;
                                sl[N + pos] = l;
                            } else {
                                sh_over = 1;
                            }
                        };
                        sweep_row(stage, [&](const float4 q, int v0) {
                            // a vector whose largest value is at or below the floor is skipped
                            const float m4 = fmaxf(fmaxf(q.x, q.y), fmaxf(q.z, q.w));
                            if (!(m4 > floor_lp)) return;   // (NaN is not finite: never a candidate)
                            stage(v0, q.x);
                            stage(v0 + 1, q.y);
                            stage(v0 + 2, q.z);
                            stage(v0 + 3, q.w);
                        });
                        __syncthreads();
                    }
                    const int staged = sh_n;
                    over = sh_over != 0;
                    __syncthreads();
                    if (!over) {
                        if (staged > 0) merge_stage(staged);
                        break;
                    }
                    for (int i = N + tid; i < sort_n2; i += NT) { sh[i] = 0; sl[i] = 0; }
                    __syncthreads();
                }
                if (!over) continue;
                // More winners than the staging room: drop the stage and sweep
                // the row again in chunks of at most `room` values, merging the
                // stage after each chunk (G only improves; each value is seen
                // once, so nothing is staged twice).
                for (int i = N + tid; i < sort_n2; i += NT) { sh[i] = 0; sl[i] = 0; }
                __syncthreads();
                const int chunk = (room / NT) * NT;
                for (int base = 0; base < V; base += chunk) {
                    const uint64_t gh = sh[N - 1], gl = sl[N - 1];
                    const float floor_lp = floor_of(gh);
                    if (tid == 0) sh_n = 0;
                    __syncthreads();
                    for (int v = base + tid; v < base + chunk && v < V; v += NT) {
                        uint64_t l = 0;
                        const uint64_t h = winner(v, lp_at(p, row + v), floor_lp, gh, gl, l);
                        if (!h) continue;
                        const int pos = atomicAdd(&sh_n, 1);
                        sh[N + pos] = h;
                        sl[N + pos] = l;
                    }
                    __syncthreads();
                    const int st = sh_n;
                    __syncthreads();
                    if (st > 0) merge_stage(st);
                }
            }
        }

        // Outputs of step t and the beam state update.
        const bool want_pool = p.pool_scores != nullptr;
        for (int j = tid; j < N; j += NT) {
            const uint64_t h = sh[j];
            const uint64_t l = sl[j];
            int parent = -1, token = -1, len = 0, flp = 0;
            float rank = -INFINITY, raw = -INFINITY;
            if (h != 0) {
                parent = cand_parent(l);
                token = cand_token(l);
                rank = cand_rank(h);
                raw = cand_raw(h);
                const bool carry = use_eos && ended[parent];
                len = carry ? (prev_len[parent] < 1 ? 1 : prev_len[parent]) : prev_len[parent] + 1;
                flp = carry ? 0 : 1;
            }
            if (want_pool && j < P) {
                const int64_t o = d.pool_offset + static_cast<int64_t>(t) * d.pool_t_stride + j;
                p.pool_parents[o] = parent;
                p.pool_tokens[o] = token;
                p.pool_lengths[o] = len;
                p.pool_raw_scores[o] = raw;
                p.pool_scores[o] = rank;
                if (p.pool_from_logprob) p.pool_from_logprob[o] = static_cast<uint8_t>(flp);
            }
            if (j < K) {
                const int64_t o = d.sel_offset + static_cast<int64_t>(t) * d.sel_t_stride + j;
                p.parents[o] = parent;
                p.tokens[o] = token;
                p.lengths[o] = len;
                if (p.raw_scores) p.raw_scores[o] = raw;
                if (p.scores) p.scores[o] = rank;
                p.from_logprob[o] = static_cast<uint8_t>(flp);
                next_raw[j] = raw;
                next_len[j] = len;
                ended_next[j] = (parent >= 0) ? ((ended[parent] != 0) || (use_eos && token == d.eos)) : 0;
            }
        }
        __syncthreads();
        for (int k = tid; k < K; k += NT) {
            prev_raw[k] = next_raw[k];
            prev_len[k] = next_len[k];
            ended[k] = ended_next[k];
        }
    }
    __syncthreads();
    if (t_stop < T) {   // more steps follow in a later call: keep the state
        if (state && !beams) {
            for (int k = tid; k < K; k += NT) {
                state[k] = prev_raw[k];
                state[seq_K + k] = __int_as_float(prev_len[k]);
                state[2 * seq_K + k] = __int_as_float(ended[k]);
                state[3 * seq_K + k] = __int_as_float(0);
            }
        }
        return true;
    }
    // Finalisation (src/differentiable_beam.cpp:1661-1667): a division.
    for (int k = tid; k < K; k += NT) {
        const int len = prev_len[k] < 1 ? 1 : prev_len[k];
        const int64_t o = d.final_offset + k;
        if (p.final_raw_scores) p.final_raw_scores[o] = prev_raw[k];
        if (p.final_scores) p.final_scores[o] = __fdiv_rn(prev_raw[k], p.pen[len]);
    }
    return true;
}

template <int NT, int PER>
__global__ void __launch_bounds__(NT, 1) list_merge_kernel(DecodeParams p, int seq_K, int sel_cap, int pf_cap) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int e = blockIdx.x;
    float* state = p.merge_state ? p.merge_state + static_cast<int64_t>(e) * 4 * seq_K : nullptr;
    unsigned char* pfb = pf_cap > 0 ? smem + align16(list_merge_smem(NT, sel_cap, seq_K)) : nullptr;
    if (pfb && threadIdx.x == 0) *reinterpret_cast<int*>(pfb) = 0;   // (published by the body's first barrier)
    list_merge_body<NT, PER>(p, e, p.t_begin > 0 ? p.t_begin : 0, p.t_end, state, seq_K, sel_cap, smem, nullptr,
                             nullptr, true, pfb, pf_cap);
}

// ---------------------------------------------------------------------------
// 3. Fused decode of a uniform batch without sequence constraints: ONE
//    cooperative launch (every CTA resident at once) in which CTAs
//    [0, merge_ctas) run the step merge and all others run the row scan.
//    The scan claims rows step by step across the examples (step-major) and
//    counts each finished row in step_done[e * T + t]; a merge CTA starts
//    step t of its example once that counter reaches K (a bounded wait,
//    which reports a timeout instead of hanging), so the T dependent merge
//    steps run while later steps are still being scanned and only the last
//    step's merge follows the scan. With fewer merge CTAs than examples a
//    CTA merges its examples one step at a time in turn, their beams kept in
//    merge_state. Merge CTAs write no output when the validation kernel
//    (queued before this launch) flagged any example; the host then
//    reports the error.
// ---------------------------------------------------------------------------
template <int PER>
__global__ void __launch_bounds__(kFusedThreads, 1) fused_decode_kernel(DecodeParams p, int capw, int seq_K,
                                                                      int sel_cap, int merge_ctas,
                                                                      unsigned int* step_done, int pf_cap) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    if (static_cast<int>(blockIdx.x) >= merge_ctas) {
        row_scan_body<false, true>(p, capw, 1, smem_raw, step_done);
        return;
    }
    __shared__ int sh_bad;
    if (threadIdx.x == 0) {
        int bad = 0;
        if (p.validate_inputs)
            for (int b = 0; b < p.B; ++b) bad |= p.status[b];
        sh_bad = bad;
    }
    __syncthreads();
    if (sh_bad) return;
    const int T = p.desc[0].T;
    // after the merge arrays: each example's beams (examples in turn), then
    // each example's prefetch block
    const int per_cta = (p.B + merge_ctas - 1) / merge_ctas;
    const size_t beams_at = align16(list_merge_smem(kFusedThreads, sel_cap, seq_K));
    const size_t pf_at = beams_at + align16(static_cast<size_t>(per_cta > 1 ? per_cta : 0) * 3 * seq_K * sizeof(float));
    const size_t pf_stride = merge_prefetch_bytes(pf_cap, seq_K);
    if (pf_cap > 0 && threadIdx.x == 0)
        for (int j = 0; j < per_cta; ++j) *reinterpret_cast<int*>(smem_raw + pf_at + j * pf_stride) = 0;
    auto pfb_of = [&](int j) { return pf_cap > 0 ? smem_raw + pf_at + j * pf_stride : nullptr; };
    if (merge_ctas >= p.B) {
        list_merge_body<kFusedThreads, PER>(p, blockIdx.x, 0, T, nullptr, seq_K, sel_cap, smem_raw, step_done,
                                            nullptr, true, pfb_of(0), pf_cap);
        return;
    }
    // examples in turn, one step at a time, each one's beams in shared memory
    float* beams_area = reinterpret_cast<float*>(smem_raw + beams_at);
    for (int t = 0; t < T; ++t) {
        int j = 0;
        for (int e = blockIdx.x; e < p.B; e += merge_ctas, ++j) {
            float* beams = beams_area + static_cast<size_t>(j) * 3 * seq_K;
            if (!list_merge_body<kFusedThreads, PER>(p, e, t, t + 1, nullptr, seq_K, sel_cap, smem_raw, step_done, beams,
                                                     t == 0 && j == 0, pfb_of(j), pf_cap))
                return;
        }
    }
}

// ---------------------------------------------------------------------------
// 2b. Step merge by ranking (no repetition penalty, no n-gram blocking).
//
// For a fixed parent the candidate key (rank, raw) is a monotone function of
// the log-prob, so it is non-increasing along the parent's row list (lp desc,
// token asc). The position of a candidate in the step's order is therefore the
// number of better candidates summed over the K row lists, each count a
// binary search on (rank, raw); equal (rank, raw) keys break ties by parent,
// then by token within one list (an equal run can hold several tokens when
// rounding maps distinct lps to one raw). Every candidate whose position is
// below N writes itself to that slot: two block barriers per step instead of
// a bitonic sort. Row lists of upcoming steps are staged into a shared ring
// with cp.async while the current step runs, so the step's critical path has
// no global-memory load.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async_8(void* smem_dst, const void* gsrc) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(s), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_4(void* smem_dst, const void* gsrc) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(s), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Waits until at most n (0..7) committed groups of this thread are pending.
__device__ __forceinline__ void cp_async_wait_pending(int n) {
    switch (n) {
        case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
        case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
        case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
        case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
        case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
        case 5: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
        case 6: asm volatile("cp.async.wait_group 6;" ::: "memory"); break;
        default: asm volatile("cp.async.wait_group 7;" ::: "memory"); break;
    }
}

constexpr int kMergeRingMax = 8;       // steps of row lists staged ahead (ring slots)
constexpr int kRescanChunk = 2048;     // log-probs per rescan chunk
constexpr int kMergeRankThreads = 1024;

// One commit group per call (empty beyond the last step) so group counting
// stays uniform across steps.
__device__ __forceinline__ void merge_stage_step(const DecodeParams& p, const ExampleDesc& d, int t, int slot,
                                                 uint64_t* ring_l, int* ring_c, float* ring_b) {
    if (t < d.T) {
        const int K = d.K, C = d.C;
        const int KC = K * C;
        const uint64_t* src = p.lists + d.list_offset + static_cast<int64_t>(t) * KC;
        uint64_t* dst = ring_l + static_cast<int64_t>(slot) * KC;
        for (int i = threadIdx.x; i < KC; i += blockDim.x) cp_async_8(dst + i, src + i);
        const int64_t row0 = d.row_begin + static_cast<int64_t>(t) * K;
        for (int k = threadIdx.x; k < K; k += blockDim.x) {
            cp_async_4(ring_c + slot * K + k, p.list_count + row0 + k);
            cp_async_4(ring_b + slot * K + k, p.list_bound + row0 + k);
        }
    }
    cp_async_commit();
}

// Rare path of the ranking merge: rescan the unproven rows of step t from HBM,
// merging every dropped candidate that beats the current N-th. Called by all
// threads of the block.
__device__ void rank_merge_rescan(const DecodeParams& p, const ExampleDesc& d, int t, const float* beam_raw,
                                  const int* beam_ended, const float* beam_inv, const uint64_t* L, const int* cnt,
                                  const float* bnd, uint64_t* cur_hi, uint64_t* cur_lo, uint64_t* st_hi,
                                  uint64_t* st_lo, int* stage_count) {
    const int K = d.K, C = d.C, N = d.N;
    const int V = p.V;
    const int tid = threadIdx.x;
    const int NT = blockDim.x;
    const bool has_eos = d.eos >= 0;
    int& sh_stage = *stage_count;
    // Rare path: rescan the unproven rows from HBM, merging every
    // dropped candidate that beats the current N-th.
    for (int j = tid; j < N; j += NT) { st_hi[j] = cur_hi[j]; st_lo[j] = cur_lo[j]; }
    __syncthreads();
    const int forced = d.forced ? d.forced[t] : -1;
    const bool eos_blocked = has_eos && (t + 1) < d.min_length;
    for (int k = 0; k < K; ++k) {
        const float pr = beam_raw[k];
        if (!isfinite(pr) || (has_eos && beam_ended[k])) continue;
        const float b = bnd[k];
        if (!(b > -INFINITY)) continue;
        const float raw_u = __fadd_rn(pr, b);
        if (raw_u == -INFINITY) continue;
        const float inv = beam_inv[k];
        {
            const uint64_t gh = st_hi[N - 1];
            const uint64_t uh = cand_hi(__fmul_rn(raw_u, inv), raw_u);
            const bool safe = gh != 0 && (gh > uh || (gh == uh && cand_parent(st_lo[N - 1]) < k));
            if (safe) continue;   // uniform: every thread reads the same staged top-N
        }
        if (tid == 0 && p.counters) atomicAdd(p.counters + 1, 1ull);
        const int64_t row = d.x_offset + (static_cast<int64_t>(t) * d.k_stride + k) * V;
        const uint64_t last = L[k * C + cnt[k] - 1];
        const float m_lp = list_lp(last);
        const int m_tok = list_token(last);
        for (int base = 0; base < V; base += kRescanChunk) {
            const uint64_t gh = st_hi[N - 1];
            const uint64_t gl = st_lo[N - 1];
            for (int v = base + tid; v < base + kRescanChunk && v < V; v += NT) {
                if (forced >= 0 && v != forced) continue;
                if (d.banned && d.banned[v]) continue;
                if (eos_blocked && v == d.eos) continue;
                if (p.row_allow && !p.row_allow[static_cast<int64_t>(k) * V + v]) continue;
                const float lp = lp_at(p, row + v);
                if (!isfinite(lp)) continue;
                const float lpc = __fadd_rn(lp, 0.0f);
                if (lpc > m_lp || (lpc == m_lp && v <= m_tok)) continue;   // already listed
                const float raw = __fadd_rn(pr, lp);
                if (raw == -INFINITY) continue;
                const uint64_t h = cand_hi(__fmul_rn(raw, inv), raw);
                const uint64_t l = cand_lo(k, v);
                if (key2_less(gh, gl, h, l)) {
                    const int pos = atomicAdd(&sh_stage, 1);
                    st_hi[N + pos] = h;
                    st_lo[N + pos] = l;
                }
            }
            __syncthreads();
            const int staged = sh_stage;
            __syncthreads();   // every thread holds the count before the next chunk stages
            if (staged > 0) {
                block_sort_desc_u128(st_hi, st_lo, N + staged);
                if (tid == 0) sh_stage = 0;
                __syncthreads();
            }
        }
    }
    for (int j = tid; j < N; j += NT) { cur_hi[j] = st_hi[j]; cur_lo[j] = st_lo[j]; }
    __syncthreads();
}

// Lanes that rank one candidate together; lane l counts lists l, l + W, ...
__device__ __forceinline__ int rank_lanes(int K) {
    int w = 1;
    while (w < K && w < 32) w <<= 1;
    return w;
}

__global__ void __launch_bounds__(kMergeRankThreads) step_merge_rank_kernel(DecodeParams p, int ring_steps,
                                                                            int max_K, int max_C, int max_N,
                                                                            int tab_n) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int e = blockIdx.x;
    const ExampleDesc d = p.desc[e];
    const int K = d.K, C = d.C, N = d.N, T = d.T, P = d.P;
    const int tid = threadIdx.x;
    const int NT = blockDim.x;
    const int R = ring_steps;
    const bool has_eos = d.eos >= 0;

    // Layout (sized by the call's largest K, C, N so every example fits).
    uint64_t* ring_l = reinterpret_cast<uint64_t*>(smem);                    // [R][K*C]
    uint64_t* top_hi = ring_l + static_cast<int64_t>(R) * max_K * max_C;   // [2][N]
    uint64_t* top_lo = top_hi + 2 * max_N;                                   // [2][N]
    uint64_t* st_hi = top_lo + 2 * max_N;                                    // [N + chunk]
    uint64_t* st_lo = st_hi + (max_N + kRescanChunk);                        // [N + chunk]
    uint64_t* carry_base = st_lo + (max_N + kRescanChunk);                   // [2][K]
    float* f_base = reinterpret_cast<float*>(carry_base + 2 * max_K);
    float* ring_b = f_base;                                                   // [R][K]
    float* raw_base = ring_b + R * max_K;                                     // [2][K]
    float* inv_base = raw_base + 2 * max_K;                                   // [2][K]
    float* tab_pen = inv_base + 2 * max_K;                                    // [tab_n]
    float* tab_inv = tab_pen + tab_n;                                         // [tab_n]
    int* ring_c = reinterpret_cast<int*>(tab_inv + tab_n);                   // [R][K]
    int* len_base = ring_c + R * max_K;                                       // [2][K]
    int* end_base = len_base + 2 * max_K;                                     // [2][K]
    __shared__ int sh_stage;

    // Length-penalty tables: shared copies when they fit, else global.
    for (int i = tid; i < tab_n; i += NT) {
        tab_pen[i] = p.pen[i];
        tab_inv[i] = p.inv_pen[i];
    }
    const float* pen = tab_n > 0 ? tab_pen : p.pen;
    const float* inv_pen = tab_n > 0 ? tab_inv : p.inv_pen;

    // Beam state and top-N slots are double buffered; cb / tb select the
    // current halves (offsets, to keep the per-thread pointer count low).
    int cb = 0;   // 0 or max_K
    int tb = 0;   // 0 or max_N

    for (int k = tid; k < K; k += NT) {
        raw_base[cb + k] = (k == 0) ? 0.0f : -INFINITY;
        len_base[cb + k] = 0;
        end_base[cb + k] = 0;
        inv_base[cb + k] = p.inv_pen[1];
        carry_base[cb + k] = 0;
    }
    for (int j = tid; j < N; j += NT) {
        top_hi[tb + j] = 0; top_lo[tb + j] = 0;
        top_hi[(max_N - tb) + j] = 0; top_lo[(max_N - tb) + j] = 0;
    }
    if (tid == 0) sh_stage = 0;
    for (int s = 0; s < R - 1; ++s) merge_stage_step(p, d, s, s, ring_l, ring_c, ring_b);

    const int W = rank_lanes(K);
    const int lane = tid & (W - 1);
    const int groups = NT / W;
    const int grp = tid / W;
    const unsigned wmask = 0xFFFFFFFFu;
    // candidates: K*C listed entries, then one bound probe per row
    const int ncand = K * C + K;

    for (int t = 0; t < T; ++t) {
        const int slot = t % R;
        cp_async_wait_pending(R - 2);
        __syncthreads();   // (a) lists of step t, beam state and cleared slots visible
        merge_stage_step(p, d, t + R - 1, (t + R - 1) % R, ring_l, ring_c, ring_b);

        const uint64_t* L = ring_l + static_cast<int64_t>(slot) * K * C;
        const int* cnt = ring_c + slot * K;
        const float* bnd = ring_b + slot * K;
        int unsafe = 0;
        // Every listed entry is a candidate: an entry past position N can
        // still place when it shares (rank, raw) with earlier entries and has
        // a lower token. The bound probe of row k asks whether at least N
        // candidates beat every entry the scan dropped from row k (which all
        // have lp <= bound, hence a key at most U = (rank(bound), raw(bound))
        // and lose ties to lower parents only); if not the row is rescanned.
        for (int base = 0; base < ncand; base += groups) {
            const int c = base + grp;
            bool active = false, probe = false;
            int k = 0, ctok = 0;
            uint64_t ch = 0;
            if (c < K * C) {
                k = c / C;
                const int i = c - k * C;
                const float pr = raw_base[cb + k];
                if (isfinite(pr)) {
                    if (has_eos && end_base[cb + k]) {
                        if (i == 0) {
                            active = true;
                            ch = carry_base[cb + k];
                            ctok = d.eos;
                        }
                    } else if (i < cnt[k]) {
                        const uint64_t key = L[k * C + i];
                        const float raw = __fadd_rn(pr, list_lp(key));
                        if (raw != -INFINITY) {
                            active = true;
                            ch = cand_hi(__fmul_rn(raw, inv_base[cb + k]), raw);
                            ctok = list_token(key);
                        }
                    }
                }
            } else if (c < ncand) {
                k = c - K * C;
                const float pr = raw_base[cb + k];
                if (isfinite(pr) && !(has_eos && end_base[cb + k])) {
                    const float b = bnd[k];
                    if (b > -INFINITY) {
                        const float raw_u = __fadd_rn(pr, b);
                        if (raw_u != -INFINITY) {
                            active = true;
                            probe = true;
                            ch = cand_hi(__fmul_rn(raw_u, inv_base[cb + k]), raw_u);
                        }
                    }
                }
            }
            int r = 0;
            if (active) {
                for (int k2 = lane; k2 < K && r < N; k2 += W) {
                    const float p2 = raw_base[cb + k2];
                    if (!isfinite(p2)) continue;
                    if (has_eos && end_base[cb + k2]) {
                        const uint64_t h2 = carry_base[cb + k2];
                        r += (h2 > ch || (h2 == ch && k2 < k)) ? 1 : 0;
                        continue;
                    }
                    const uint64_t* L2 = L + k2 * C;
                    const float inv2 = inv_base[cb + k2];
                    const int n2 = cnt[k2];
                    int lo = 0, hi = n2;
                    while (lo < hi) {
                        const int mid = (lo + hi) >> 1;
                        const float raw2 = __fadd_rn(p2, list_lp(L2[mid]));
                        const uint64_t h2 = cand_hi(__fmul_rn(raw2, inv2), raw2);
                        if (h2 > ch) lo = mid + 1;
                        else hi = mid;
                    }
                    r += lo;
                    if (k2 < k || (k2 == k && !probe)) {
                        // equal (rank, raw): lower parents win; within the
                        // same parent the lower token wins
                        for (int j = lo; j < n2 && r < N; ++j) {
                            const uint64_t key2 = L2[j];
                            const float raw2 = __fadd_rn(p2, list_lp(key2));
                            if (cand_hi(__fmul_rn(raw2, inv2), raw2) != ch) break;
                            if (k2 < k || list_token(key2) < ctok) ++r;
                        }
                    }
                }
            }
            for (int o = W >> 1; o > 0; o >>= 1) r += __shfl_xor_sync(wmask, r, o);
            if (active && lane == 0 && r < N) {
                if (probe) {
                    unsafe = 1;
                } else {
                    top_hi[tb + r] = ch;
                    top_lo[tb + r] = cand_lo(k, ctok);
                }
            }
        }
        // (b) top-N of step t in the current slots; any unproven row
        const bool any_unsafe = __syncthreads_or(unsafe) != 0;

        if (any_unsafe)
            rank_merge_rescan(p, d, t, raw_base + cb, end_base + cb, inv_base + cb, L, cnt, bnd, top_hi + tb,
                              top_lo + tb, st_hi, st_lo, &sh_stage);

        // Outputs of step t, next beam state, and the cleared slots of step t+1.
        const bool want_pool = p.pool_scores != nullptr;
        for (int j = tid; j < N; j += NT) {
            const uint64_t h = top_hi[tb + j];
            const uint64_t l = top_lo[tb + j];
            int parent = -1, token = -1, len = 0, flp = 0;
            float rank = -INFINITY, raw = -INFINITY;
            bool carry = false;
            if (h != 0) {
                parent = cand_parent(l);
                token = cand_token(l);
                rank = cand_rank(h);
                raw = cand_raw(h);
                carry = has_eos && end_base[cb + parent];
                len = carry ? (len_base[cb + parent] < 1 ? 1 : len_base[cb + parent]) : len_base[cb + parent] + 1;
                flp = carry ? 0 : 1;
            }
            if (want_pool && j < P) {
                const int64_t o = d.pool_offset + static_cast<int64_t>(t) * d.pool_t_stride + j;
                p.pool_parents[o] = parent;
                p.pool_tokens[o] = token;
                p.pool_lengths[o] = len;
                p.pool_raw_scores[o] = raw;
                p.pool_scores[o] = rank;
                if (p.pool_from_logprob) p.pool_from_logprob[o] = static_cast<uint8_t>(flp);
            }
            if (j < K) {
                const int64_t o = d.sel_offset + static_cast<int64_t>(t) * d.sel_t_stride + j;
                p.parents[o] = parent;
                p.tokens[o] = token;
                p.lengths[o] = len;
                if (p.raw_scores) p.raw_scores[o] = raw;
                if (p.scores) p.scores[o] = rank;
                p.from_logprob[o] = static_cast<uint8_t>(flp);
                const int ended = (parent >= 0) ? ((carry || (has_eos && token == d.eos)) ? 1 : 0) : 0;
                raw_base[(max_K - cb) + j] = raw;
                len_base[(max_K - cb) + j] = len;
                end_base[(max_K - cb) + j] = ended;
                inv_base[(max_K - cb) + j] = inv_pen[len + 1];
                uint64_t ck = 0;
                if (ended && isfinite(raw)) {
                    const int cl = len < 1 ? 1 : len;
                    ck = cand_hi(__fdiv_rn(raw, pen[cl]), raw);
                }
                carry_base[(max_K - cb) + j] = ck;
            }
            top_hi[(max_N - tb) + j] = 0;
            top_lo[(max_N - tb) + j] = 0;
        }
        cb = max_K - cb;
        tb = max_N - tb;
    }
    cp_async_wait_pending(0);
    __syncthreads();
    // Finalisation (src/differentiable_beam.cpp:1661-1667): a division, not
    // a multiply by the reciprocal.
    for (int k = tid; k < K; k += NT) {
        const int len = len_base[cb + k] < 1 ? 1 : len_base[cb + k];
        const int64_t o = d.final_offset + k;
        if (p.final_raw_scores) p.final_raw_scores[o] = raw_base[cb + k];
        if (p.final_scores) p.final_scores[o] = __fdiv_rn(raw_base[cb + k], pen[len]);
    }
}

// ---------------------------------------------------------------------------
// 3. Weights: selected softmax (softmax_selected_scalar, :410-442) and relaxed
//    pool weights (soft_topk_inclusion, :1333-1386). One warp per step.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float safe_exp_dev(float x) {
    const float hi = 88.3762626647949f;
    x = (-hi < x) ? x : -hi;
    x = (x < hi) ? x : hi;
    return expf(x);
}
__device__ __forceinline__ float sigmoid_dev(float x) {
    if (x >= 0.0f) {
        const float e = safe_exp_dev(-x);
        return __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
    }
    const float e = safe_exp_dev(x);
    return __fdiv_rn(e, __fadd_rn(1.0f, e));
}

template <int MAXP>
__global__ void weights_kernel(DecodeParams p, int max_T) {
    constexpr int kPer = (MAXP + 31) / 32;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int e = warp / max_T;
    const int t = warp - e * max_T;
    if (e >= p.B) return;
    const ExampleDesc d = p.desc[e];
    if (t >= d.T) return;
    const float guard = -1.0e30f;
    if (p.weights && p.scores) {
        const int K = d.K;
        const int64_t o = d.sel_offset + static_cast<int64_t>(t) * d.sel_t_stride;
        const float temp = p.selected_temperature;
        float mx = -INFINITY;
        for (int i = lane; i < K; i += 32) {
            const float sc = p.scores[o + i];
            if (sc > guard) mx = fmaxf(mx, __fdiv_rn(sc, temp));
        }
        mx = warp_max(mx);
        if (!isfinite(mx)) {
            for (int i = lane; i < K; i += 32) p.weights[o + i] = 0.0f;
        } else {
            float sum = 0.0f;
            for (int i = lane; i < K; i += 32) {
                const float sc = p.scores[o + i];
                if (sc > guard) sum = __fadd_rn(sum, safe_exp_dev(__fsub_rn(__fdiv_rn(sc, temp), mx)));
            }
            sum = warp_sum(sum);
            if (!(sum > 0.0f) || !isfinite(sum)) {
                for (int i = lane; i < K; i += 32) p.weights[o + i] = 0.0f;
            } else {
                const float inv = __fdiv_rn(1.0f, sum);
                for (int i = lane; i < K; i += 32) {
                    const float sc = p.scores[o + i];
                    float w = 0.0f;
                    if (sc > guard) w = __fmul_rn(safe_exp_dev(__fsub_rn(__fdiv_rn(sc, temp), mx)), inv);
                    p.weights[o + i] = w;
                }
            }
        }
    }
    if (p.relaxed_weights && p.pool_scores) {
        const int P = d.P;
        const int target = d.K;
        const int64_t o = d.pool_offset + static_cast<int64_t>(t) * d.pool_t_stride;
        const float temp = p.soft_topk_temperature;
        const float tol = p.soft_topk_tolerance;
        float sv[kPer];
        int active = 0;
        float mn = INFINITY, mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int i = lane + 32 * j;
            sv[j] = (i < P) ? p.pool_scores[o + i] : -INFINITY;
            if (sv[j] > guard) {
                ++active;
                mn = fminf(mn, sv[j]);
                mx = fmaxf(mx, sv[j]);
            }
        }
        active = warp_isum(active);
        mn = warp_min(mn);
        mx = warp_max(mx);
        float out[kPer];
#pragma unroll
        for (int j = 0; j < kPer; ++j) out[j] = 0.0f;
        if (active > 0 && target > 0) {
            if (target >= active) {
#pragma unroll
                for (int j = 0; j < kPer; ++j) out[j] = (sv[j] > guard) ? 1.0f : 0.0f;
            } else {
                float lo = __fsub_rn(mn, __fmul_rn(80.0f, temp));
                float hi = __fadd_rn(mx, __fmul_rn(80.0f, temp));
                for (int it = 0; it < p.soft_topk_max_iters; ++it) {
                    const float mid = __fmul_rn(0.5f, __fadd_rn(lo, hi));
                    float sum = 0.0f;
#pragma unroll
                    for (int j = 0; j < kPer; ++j)
                        if (sv[j] > guard) sum = __fadd_rn(sum, sigmoid_dev(__fdiv_rn(__fsub_rn(sv[j], mid), temp)));
                    sum = warp_sum(sum);
                    const float err = __fsub_rn(sum, static_cast<float>(target));
                    const float amid = fabsf(mid);
                    if (fabsf(err) <= tol || fabsf(__fsub_rn(hi, lo)) <= __fmul_rn(tol, fmaxf(1.0f, amid))) {
                        lo = hi = mid;
                        break;
                    }
                    if (err > 0.0f) lo = mid; else hi = mid;
                }
                const float theta = __fmul_rn(0.5f, __fadd_rn(lo, hi));
#pragma unroll
                for (int j = 0; j < kPer; ++j)
                    out[j] = (sv[j] > guard) ? sigmoid_dev(__fdiv_rn(__fsub_rn(sv[j], theta), temp)) : 0.0f;
            }
        }
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int i = lane + 32 * j;
            if (i < P) p.relaxed_weights[o + i] = out[j];
        }
    }
}

// ---------------------------------------------------------------------------
// 4. Surrogate backward (backward_sparse / backward, :1674-1791). One CTA per
//    example walks t = T-1 .. 0. prev_raw_grad is accumulated per parent in
//    the reference's order (selected k ascending, then pool p ascending).
// ---------------------------------------------------------------------------
// The per-example body; `d`, the 1/gnmt table and the [B, max_T] step-count
// scratch come from the caller so the no-allocation variant below can supply
// them without device metadata.
__device__ __forceinline__ void backward_example(const BackwardParams& p, const ExampleDesc& d, int e,
                                                 const float* __restrict__ inv_pen, int32_t* step_counts,
                                                 int sparse, int max_K, int max_P) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int K = d.K, T = d.T, P = d.P;
    const int64_t V = p.V;
    const int tid = threadIdx.x;
    const int NT = blockDim.x;
    float* next_g = reinterpret_cast<float*>(smem);
    float* prev_g = next_g + max_K;
    float* sel_draw = prev_g + max_K;
    float* pool_draw = sel_draw + max_K;
    int* sel_parent = reinterpret_cast<int*>(pool_draw + max_P);
    int* pool_parent = sel_parent + max_K;
    uint64_t* ent_key = reinterpret_cast<uint64_t*>(pool_parent + max_P);
    float* ent_val = reinterpret_cast<float*>(ent_key + (max_K + max_P));
    __shared__ float sh_dot;
    __shared__ float sh_center;
    __shared__ int sh_relax;
    __shared__ int sh_n;

    for (int k = tid; k < K; k += NT) next_g[k] = 0.0f;
    __syncthreads();
    const float inv_temp_soft = __fdiv_rn(1.0f, p.soft_topk_temperature);
    for (int t = T - 1; t >= 0; --t) {
        const int64_t so = d.sel_offset + static_cast<int64_t>(t) * d.sel_t_stride;
        const int64_t po = d.pool_offset + static_cast<int64_t>(t) * d.pool_t_stride;
        if (tid == 0) {
            sh_n = 0;
            float dot = 0.0f;
            if (p.grad_selected) {
                for (int k = 0; k < K; ++k)
                    dot = __fadd_rn(dot, __fmul_rn(p.weights[so + k], p.grad_selected[so + k]));
            }
            sh_dot = dot;
            sh_relax = 0;
            if (p.grad_relaxed) {
                float denom = 0.0f, numer = 0.0f;
                for (int q = 0; q < P; ++q) {
                    const float w = p.relaxed_weights[po + q];
                    const float a = __fmul_rn(w, __fsub_rn(1.0f, w));
                    denom = __fadd_rn(denom, a);
                    numer = __fadd_rn(numer, __fmul_rn(p.grad_relaxed[po + q], a));
                }
                if (denom > 1.0e-12f) {
                    sh_relax = 1;
                    sh_center = __fdiv_rn(numer, denom);
                }
            }
        }
        __syncthreads();
        // selected slots
        for (int k = tid; k < K; k += NT) {
            const int parent = p.parents[so + k];
            float draw = 0.0f;
            if (parent >= 0) {
                float drank = 0.0f;
                if (p.grad_selected) {
                    const float w = p.weights[so + k];
                    drank = __fadd_rn(drank, __fdiv_rn(__fmul_rn(w, __fsub_rn(p.grad_selected[so + k], sh_dot)),
                                                       p.selected_temperature));
                }
                if (p.grad_final && t == T - 1) drank = __fadd_rn(drank, p.grad_final[d.final_offset + k]);
                const int len = p.lengths[so + k] < 1 ? 1 : p.lengths[so + k];
                draw = __fadd_rn(next_g[k], __fmul_rn(drank, inv_pen[len]));
                const int token = p.tokens[so + k];
                if (draw != 0.0f && p.from_logprob[so + k] && token >= 0) {
                    const int64_t gi = (static_cast<int64_t>(t) * K + parent) * V + token;
                    if (sparse) {
                        const int pos = atomicAdd(&sh_n, 1);
                        ent_key[pos] = ~((static_cast<uint64_t>(gi) << 12) | static_cast<uint64_t>(pos));
                        ent_val[pos] = draw;
                    } else {
                        p.grad_dense[d.grad_offset + gi] = draw;
                    }
                }
            }
            sel_parent[k] = (parent >= 0 && draw != 0.0f) ? parent : -1;
            sel_draw[k] = draw;
        }
        __syncthreads();
        // relaxed pool
        if (sh_relax) {
            const float center = sh_center;
            for (int q = tid; q < P; q += NT) {
                const int parent = p.pool_parents[po + q];
                float draw = 0.0f;
                if (parent >= 0) {
                    const float w = p.relaxed_weights[po + q];
                    const float a = __fmul_rn(w, __fsub_rn(1.0f, w));
                    const float drank = __fmul_rn(__fmul_rn(a, inv_temp_soft), __fsub_rn(p.grad_relaxed[po + q], center));
                    if (drank != 0.0f) {
                        const int len = p.pool_lengths[po + q] < 1 ? 1 : p.pool_lengths[po + q];
                        draw = __fmul_rn(drank, inv_pen[len]);
                        const int token = p.pool_tokens[po + q];
                        if (draw != 0.0f && p.pool_from_logprob[po + q] && token >= 0) {
                            const int64_t gi = (static_cast<int64_t>(t) * K + parent) * V + token;
                            if (sparse) {
                                const int pos = atomicAdd(&sh_n, 1);
                                ent_key[pos] = ~((static_cast<uint64_t>(gi) << 12) | static_cast<uint64_t>(pos));
                                ent_val[pos] = draw;
                            } else {
                                atomicAdd(p.grad_dense + d.grad_offset + gi, draw);
                            }
                        }
                    }
                }
                pool_parent[q] = (parent >= 0 && draw != 0.0f) ? parent : -1;
                pool_draw[q] = draw;
            }
        }
        __syncthreads();
        // prev_raw_grad in the reference's accumulation order
        for (int j = tid; j < K; j += NT) {
            float acc = 0.0f;
            for (int k = 0; k < K; ++k)
                if (sel_parent[k] == j) acc = __fadd_rn(acc, sel_draw[k]);
            if (sh_relax)
                for (int q = 0; q < P; ++q)
                    if (pool_parent[q] == j) acc = __fadd_rn(acc, pool_draw[q]);
            prev_g[j] = acc;
        }
        if (sparse) {
            // Sort this step's entries by index (keys hold ~(index << 12 | slot)
            // so a descending sort yields ascending indices) and merge the at
            // most two entries of one index (finalize_sparse_entries,
            // src/differentiable_beam.cpp:1908-1941).
            __syncthreads();
            const int n = sh_n;
            block_sort_desc_u64(ent_key, n);
            if (tid == 0) {
                const int64_t seg = d.sparse_offset + static_cast<int64_t>(t) * (K + P);
                int m = 0;
                for (int a = 0; a < n;) {
                    const uint64_t ka = ~ent_key[a];
                    const int64_t gi = static_cast<int64_t>(ka >> 12);
                    float sum = 0.0f;
                    int b = a;
                    while (b < n && static_cast<int64_t>((~ent_key[b]) >> 12) == gi) {
                        sum = __fadd_rn(sum, ent_val[(~ent_key[b]) & 0xFFFu]);
                        ++b;
                    }
                    p.sparse_indices[seg + m] = gi;
                    p.sparse_values[seg + m] = sum;
                    ++m;
                    a = b;
                }
                step_counts[static_cast<int64_t>(e) * p.max_T + t] = m;
            }
        }
        __syncthreads();
        for (int k = tid; k < K; k += NT) next_g[k] = prev_g[k];
        __syncthreads();
    }
    for (int k = tid; k < K; k += NT)
        if (p.grad_initial) p.grad_initial[d.final_offset + k] = next_g[k];
    if (sparse) {
        // compact the per-step segments (t ascending == index ascending)
        __syncthreads();
        int64_t off = 0;
        for (int t = 0; t < T; ++t) {
            const int m = step_counts[static_cast<int64_t>(e) * p.max_T + t];
            const int64_t src = d.sparse_offset + static_cast<int64_t>(t) * (K + P);
            const int64_t dst = d.sparse_offset + off;
            if (dst != src) {
                // read all, then write (ranges may overlap; dst < src)
                int64_t* tmp_idx = reinterpret_cast<int64_t*>(ent_key);
                for (int a = tid; a < m; a += NT) {
                    tmp_idx[a] = p.sparse_indices[src + a];
                    ent_val[a] = p.sparse_values[src + a];
                }
                __syncthreads();
                for (int a = tid; a < m; a += NT) {
                    p.sparse_indices[dst + a] = tmp_idx[a];
                    p.sparse_values[dst + a] = ent_val[a];
                }
                __syncthreads();
            }
            off += m;
        }
        if (tid == 0) p.sparse_counts[e] = off;
    }
}

__global__ void backward_kernel(BackwardParams p, int sparse, int max_K, int max_P) {
    const int e = blockIdx.x;
    const ExampleDesc d = p.desc[e];
    backward_example(p, d, e, p.inv_pen, p.step_counts, sparse, max_K, max_P);
}

// ---------------------------------------------------------------------------
// 4b. Dense surrogate backward for beams of at most 32: everything that does
//     not depend on the reverse recursion (per-step dot products and pool
//     centres, each selected slot's own rank gradient times 1/gnmt, the whole
//     relaxed-pool contribution) is computed for all steps in parallel first;
//     the recursion itself (draw = next_g[k] + own term, then the per-parent
//     sums in the reference's order: selected k ascending, then pool q
//     ascending) runs in one warp out of shared memory, lane k owning beam k.
//     The arithmetic is the same sequence of rounded operations as the block
//     kernel above. A gradient index receives at most two contributions (the
//     selected slot and the pool slot of the same candidate); both are added
//     with atomicAdd into the zeroed buffer, which is exact in either order.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) backward_sweep_kernel(BackwardParams p, int max_T, int max_K, int max_P,
                                                             int with_pool, int sparse) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int e = blockIdx.x;
    const ExampleDesc d = p.desc[e];
    const int K = d.K, T = d.T, P = d.P;
    const int64_t V = p.V;
    const int tid = threadIdx.x;
    const int NT = blockDim.x;
    float* own = reinterpret_cast<float*>(smem);                 // [T*K] drank * inv_pen[len]
    int* par = reinterpret_cast<int*>(own + max_T * max_K);      // [T*K] parent (-1 none)
    int* tok = par + max_T * max_K;                              // [T*K] token if it writes, else -1
    float* dot = reinterpret_cast<float*>(tok + max_T * max_K);  // [T]
    float* center = dot + max_T;                                 // [T]
    int* relax = reinterpret_cast<int*>(center + max_T);         // [T]
    int* ppar = relax + max_T;                                   // [T*P] pool parent with a draw, else -1
    float* pdraw = reinterpret_cast<float*>(ppar + (with_pool ? max_T * max_P : 0));  // [T*P]

    // per-step reductions, in the reference's sequential order
    for (int t = tid; t < T; t += NT) {
        const int64_t so = d.sel_offset + static_cast<int64_t>(t) * d.sel_t_stride;
        const int64_t po = d.pool_offset + static_cast<int64_t>(t) * d.pool_t_stride;
        float dt = 0.0f;
        if (p.grad_selected)
            for (int k = 0; k < K; ++k) dt = __fadd_rn(dt, __fmul_rn(p.weights[so + k], p.grad_selected[so + k]));
        dot[t] = dt;
        int rl = 0;
        float ctr = 0.0f;
        if (p.grad_relaxed) {
            float denom = 0.0f, numer = 0.0f;
            for (int q = 0; q < P; ++q) {
                const float w = p.relaxed_weights[po + q];
                const float a = __fmul_rn(w, __fsub_rn(1.0f, w));
                denom = __fadd_rn(denom, a);
                numer = __fadd_rn(numer, __fmul_rn(p.grad_relaxed[po + q], a));
            }
            if (denom > 1.0e-12f) {
                rl = 1;
                ctr = __fdiv_rn(numer, denom);
            }
        }
        relax[t] = rl;
        center[t] = ctr;
    }
    __syncthreads();
    // selected slots: the part of each draw that does not depend on next_g
    for (int idx = tid; idx < T * K; idx += NT) {
        const int t = idx / K;
        const int k = idx - t * K;
        const int64_t so = d.sel_offset + static_cast<int64_t>(t) * d.sel_t_stride;
        const int parent = p.parents[so + k];
        float m = 0.0f;
        int tk = -1;
        if (parent >= 0) {
            float drank = 0.0f;
            if (p.grad_selected) {
                const float w = p.weights[so + k];
                drank = __fadd_rn(drank, __fdiv_rn(__fmul_rn(w, __fsub_rn(p.grad_selected[so + k], dot[t])),
                                                   p.selected_temperature));
            }
            if (p.grad_final && t == T - 1) drank = __fadd_rn(drank, p.grad_final[d.final_offset + k]);
            const int len = p.lengths[so + k] < 1 ? 1 : p.lengths[so + k];
            m = __fmul_rn(drank, p.inv_pen[len]);
            const int token = p.tokens[so + k];
            if (p.from_logprob[so + k] && token >= 0) tk = token;
        }
        own[idx] = m;
        par[idx] = parent;
        tok[idx] = tk;
    }
    // relaxed pool: independent of the recursion, written now
    if (with_pool) {
        const float inv_temp_soft = __fdiv_rn(1.0f, p.soft_topk_temperature);
        for (int idx = tid; idx < T * P; idx += NT) {
            const int t = idx / P;
            const int q = idx - t * P;
            int pp = -1;
            float draw = 0.0f;
            if (relax[t]) {
                const int64_t po = d.pool_offset + static_cast<int64_t>(t) * d.pool_t_stride;
                const int parent = p.pool_parents[po + q];
                if (parent >= 0) {
                    const float w = p.relaxed_weights[po + q];
                    const float a = __fmul_rn(w, __fsub_rn(1.0f, w));
                    const float drank = __fmul_rn(__fmul_rn(a, inv_temp_soft), __fsub_rn(p.grad_relaxed[po + q], center[t]));
                    if (drank != 0.0f) {
                        const int len = p.pool_lengths[po + q] < 1 ? 1 : p.pool_lengths[po + q];
                        draw = __fmul_rn(drank, p.inv_pen[len]);
                        const int token = p.pool_tokens[po + q];
                        if (draw != 0.0f && p.pool_from_logprob[po + q] && token >= 0) {
                            const int64_t gi = (static_cast<int64_t>(t) * K + parent) * V + token;
                            atomicAdd(p.grad_dense + d.grad_offset + gi, draw);
                        }
                    }
                }
                pp = (parent >= 0 && draw != 0.0f) ? parent : -1;
            }
            ppar[idx] = pp;
            pdraw[idx] = draw;
        }
    }
    __syncthreads();
    if (tid < 32) {
        // the recursion: one warp, lane k = beam k
        const int lane = tid;
        float g = 0.0f;
        for (int t = T - 1; t >= 0; --t) {
            float draw = 0.0f;
            int sp = -1;
            if (lane < K) {
                const int idx = t * K + lane;
                const int parent = par[idx];
                if (parent >= 0) {
                    draw = __fadd_rn(g, own[idx]);
                    const int tk = tok[idx];
                    if (sparse) {
                        // keep the entry for the sparse output below
                        own[idx] = draw;
                        if (draw == 0.0f) tok[idx] = -1;
                    } else if (draw != 0.0f && tk >= 0) {
                        const int64_t gi = (static_cast<int64_t>(t) * K + parent) * V + tk;
                        if (with_pool && relax[t]) atomicAdd(p.grad_dense + d.grad_offset + gi, draw);
                        else p.grad_dense[d.grad_offset + gi] = draw;
                    }
                    if (draw != 0.0f) sp = parent;
                }
            }
            float acc = 0.0f;
            for (int k = 0; k < K; ++k) {
                const int pk = __shfl_sync(0xFFFFFFFFu, sp, k);
                const float dk = __shfl_sync(0xFFFFFFFFu, draw, k);
                if (pk == lane) acc = __fadd_rn(acc, dk);
            }
            if (with_pool && relax[t]) {
                const int* pq = ppar + t * P;
                const float* dq = pdraw + t * P;
                for (int q = 0; q < P; ++q)
                    if (pq[q] == lane) acc = __fadd_rn(acc, dq[q]);
            }
            g = acc;
        }
        if (lane < K && p.grad_initial) p.grad_initial[d.final_offset + lane] = g;
    }
    if (!sparse) return;
    // Sparse output without a relaxed-pool gradient: a step's entries are
    // its selected slots, whose (parent, token) pairs are distinct, so the
    // sorted unique indices (finalize_sparse_entries,
    // src/differentiable_beam.cpp:1908-1941) are each step's entries sorted
    // by (parent, token), steps in order. One warp sorts a step in
    // registers; one scan of the per-step counts places the steps.
    __syncthreads();
    int* step_n = relax;                           // [T] entries of step t
    int* step_off = reinterpret_cast<int*>(dot);   // [T] their first output slot
    const int lane = tid & 31;
    for (int t = tid >> 5; t < T; t += NT >> 5) {
        const int idx = t * K + lane;
        const int pa = lane < K ? par[idx] : -1;
        const int tk = lane < K ? tok[idx] : -1;
        const bool ok = pa >= 0 && tk >= 0;
        uint64_t key = ok ? (static_cast<uint64_t>(pa) << 32) | static_cast<uint32_t>(tk) : ~0ull;
        float val = lane < K ? own[idx] : 0.0f;
#pragma unroll
        for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
            for (int st = size >> 1; st > 0; st >>= 1) {
                const uint64_t ok2 = __shfl_xor_sync(0xFFFFFFFFu, key, st);
                const float ov = __shfl_xor_sync(0xFFFFFFFFu, val, st);
                const bool lower = (lane & st) == 0;
                const bool asc = (lane & size) == 0;
                if (lower == asc ? ok2 < key : ok2 > key) {
                    key = ok2;
                    val = ov;
                }
            }
        }
        const int n = __popc(__ballot_sync(0xFFFFFFFFu, ok));
        __syncwarp();
        if (lane < n) {
            par[idx] = static_cast<int>(key >> 32);
            tok[idx] = static_cast<int>(key & 0xFFFFFFFFu);
            own[idx] = val;
        }
        if (lane == 0) step_n[t] = n;
    }
    __syncthreads();
    if (tid < 32) {
        int base = 0;
        for (int t0 = 0; t0 < T; t0 += 32) {
            const int t = t0 + tid;
            const int n = t < T ? step_n[t] : 0;
            int incl = n;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
                if (tid >= o) incl += v;
            }
            if (t < T) step_off[t] = base + incl - n;
            base += __shfl_sync(0xFFFFFFFFu, incl, 31);
        }
        if (tid == 0) p.sparse_counts[e] = base;
    }
    __syncthreads();
    for (int idx = tid; idx < T * K; idx += NT) {
        const int t = idx / K;
        const int j = idx - t * K;
        if (j < step_n[t]) {
            const int64_t o = d.sparse_offset + step_off[t] + j;
            p.sparse_indices[o] = (static_cast<int64_t>(t) * K + par[idx]) * V + tok[idx];
            p.sparse_values[o] = own[idx];
        }
    }
}

// ---------------------------------------------------------------------------
// 5. Zero fill with 128-bit stores (dense gradient).
// ---------------------------------------------------------------------------
__global__ void fill_zero_kernel(float* __restrict__ dst, int64_t count) {
    const uintptr_t addr = reinterpret_cast<uintptr_t>(dst);
    int64_t h = static_cast<int64_t>(((16u - (addr & 15u)) & 15u) >> 2);
    if (h > count) h = count;
    const int64_t gtid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t gsz = static_cast<int64_t>(gridDim.x) * blockDim.x;
    if (gtid < h) dst[gtid] = 0.0f;
    const int64_t nv = (count - h) >> 2;
    float4* d4 = reinterpret_cast<float4*>(dst + h);
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int64_t i = gtid; i < nv; i += gsz) __stcs(d4 + i, z);
    const int64_t tail0 = h + 4 * nv;
    if (gtid < count - tail0) dst[tail0 + gtid] = 0.0f;
}

// Zero fill through the bulk-copy (TMA) engine: one warp per CTA zeroes a
// shared tile once and lane 0 streams it to global memory with 1-D bulk
// stores (cp.async.bulk.global.shared::cta, no multicast). A handful of
// instructions per 32 KB keeps the SM's load/store pipe free for the
// latency-bound step merge that runs beside the fill. The unaligned head and
// tail (fewer than 4 elements each) use plain stores.
constexpr int kFillTileBytes = 32 * 1024;
constexpr int kFillInFlight = 8;   // bulk groups a CTA keeps in flight

__global__ void __launch_bounds__(32, 1) fill_zero_bulk_kernel(float* __restrict__ dst, int64_t count) {
    extern __shared__ __align__(128) unsigned char zbuf[];
    const int lane = threadIdx.x;
    float4* z4 = reinterpret_cast<float4*>(zbuf);
    for (int i = lane; i < kFillTileBytes / 16; i += 32) z4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    // generic-proxy writes of the tile must be visible to the bulk engine
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    const uintptr_t addr = reinterpret_cast<uintptr_t>(dst);
    int64_t h = static_cast<int64_t>(((16u - (addr & 15u)) & 15u) >> 2);
    if (h > count) h = count;
    const int64_t body = ((count - h) >> 2) << 4;   // bytes, multiple of 16
    const int64_t tail0 = h + (body >> 2);
    if (blockIdx.x == 0) {
        if (lane < h) dst[lane] = 0.0f;
        if (lane < count - tail0) dst[tail0 + lane] = 0.0f;
    }
    if (lane == 0 && body > 0) {
        char* base = reinterpret_cast<char*>(dst + h);
        const uint32_t src = static_cast<uint32_t>(__cvta_generic_to_shared(zbuf));
        const int64_t tiles = (body + kFillTileBytes - 1) / kFillTileBytes;
        for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
            const int64_t off = tile * kFillTileBytes;
            const int64_t rem = body - off;
            const uint32_t bytes = static_cast<uint32_t>(rem < kFillTileBytes ? rem : kFillTileBytes);
            asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
                         ::"l"(base + off), "r"(src), "r"(bytes) : "memory");
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(kFillInFlight) : "memory");
        }
        // the tile must stay valid until every store has read it, and the
        // writes are complete before the CTA retires
        asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }
    __syncwarp();
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------

// cudaFuncSetAttribute / occupancy results are cached per (kernel, device):
// the runtime calls cost microseconds and the launchers run on every decode.
static std::mutex g_attr_mu;
static std::vector<std::tuple<const void*, int, size_t>> g_smem_set;
static std::vector<std::tuple<int, size_t, int>> g_row_scan_occ;
static std::vector<std::pair<const void*, int>> g_carveout_set;

// Launches queued by the launchers below (process-wide, for benchmarks).
static std::atomic<long long> g_kernel_launches{0};
static cudaError_t counted(cudaError_t err) {
    if (err == cudaSuccess) g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    return err;
}
long long kernel_launch_count() { return g_kernel_launches.load(std::memory_order_relaxed); }

static cudaError_t prefer_shared(const void* fn);

static cudaError_t ensure_dynamic_smem(const void* fn, size_t smem) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    std::lock_guard<std::mutex> lock(g_attr_mu);
    for (auto& e : g_smem_set) {
        if (std::get<0>(e) == fn && std::get<1>(e) == dev) {
            if (std::get<2>(e) >= smem) return cudaSuccess;
            err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
            if (err == cudaSuccess) std::get<2>(e) = smem;
            return err;
        }
    }
    err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (err != cudaSuccess) return err;
    err = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                               static_cast<int>(cudaSharedmemCarveoutMaxShared));
    if (err == cudaSuccess) g_smem_set.emplace_back(fn, dev, smem);
    return err;
}

// Every kernel of the engine asks for the largest shared-memory carveout. An SM
// switches carveout only when it is idle, so a kernel that left its SMs in a
// small-shared-memory configuration (the zero fill, the validator) would hold
// back a shared-memory kernel queued beside or after it until those SMs drain.
static cudaError_t prefer_shared(const void* fn) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    std::lock_guard<std::mutex> lock(g_attr_mu);
    for (auto& e : g_carveout_set)
        if (e.first == fn && e.second == dev) return cudaSuccess;
    err = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                               static_cast<int>(cudaSharedmemCarveoutMaxShared));
    if (err == cudaSuccess) g_carveout_set.emplace_back(fn, dev);
    return err;
}

cudaError_t launch_validate(const DecodeParams& p, cudaStream_t stream) {
    cudaError_t err = prefer_shared(reinterpret_cast<const void*>(validate_kernel));
    if (err != cudaSuccess) return err;
    validate_kernel<<<p.B, 1024, 0, stream>>>(p);
    return counted(cudaGetLastError());
}

// Per-warp survivor buffer: C kept + max(C, 16) appended between compactions +
// one 128-value group of appends + 8. A compaction sorts the buffer, so for
// large C it runs once per C survivors (a few times per row) rather than once
// per 16.
static int row_scan_capw(int max_C) { return max_C + (max_C > 16 ? max_C : 16) + 128 + 8; }

static size_t row_scan_smem(int capw, bool k16) {
    return static_cast<size_t>(kScanWarpsPerCta) * row_scan_warp_bytes(capw, k16);
}

cudaError_t launch_row_scan(const DecodeParams& p, int max_C, int num_sms, cudaStream_t stream, int64_t rows,
                            int speculate_mode) {
    if (rows < 0) rows = p.total_rows;
    if (rows <= 0) return cudaSuccess;
    const bool k16 = p.x16 != nullptr;
    // 16-bit rows append up to 256 values between compaction checks
    int capw = row_scan_capw(max_C) + (k16 ? 128 : 0);
    const void* fn = k16 ? reinterpret_cast<const void*>(row_scan_kernel<true>)
                         : reinterpret_cast<const void*>(row_scan_kernel<false>);
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    if (max_C > 32) {
        // Long lists: shrink the survivor buffer so that the 4 CTAs per SM
        // the launch bounds plan for fit in shared memory (more compactions,
        // but a third more warps than 3 CTAs at C = 256), when that leaves
        // room for one append group plus 32 entries above C.
        int per_sm_smem = 0, reserved = 0;
        err = cudaDeviceGetAttribute(&per_sm_smem, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
        if (err != cudaSuccess) return err;
        err = cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
        if (err != cudaSuccess) return err;
        const int per_warp = ((per_sm_smem / 4 - reserved) / kScanWarpsPerCta) & ~127;
        const int fixed = kScanStages * kScanChunkF4 * 16 + kScanStages * 8 + 256 * 4 + kSpecSlots * 8;
        const int fit = (per_warp - fixed) / 8;
        const int lowest = max_C + (k16 ? 256 : 128) + 8 + 32;
        if (fit >= lowest && fit < capw) capw = fit;
    }
    const int threads = kScanWarpsPerCta * 32;
    const size_t smem = row_scan_smem(capw, k16);
    err = ensure_dynamic_smem(fn, smem);
    if (err != cudaSuccess) return err;
    const int key = dev + (k16 ? 1 << 20 : 0);
    int per_sm = -1;
    {
        std::lock_guard<std::mutex> lock(g_attr_mu);
        for (auto& e : g_row_scan_occ)
            if (std::get<0>(e) == key && std::get<1>(e) == smem) per_sm = std::get<2>(e);
    }
    if (per_sm < 0) {
        err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem);
        if (err != cudaSuccess) return err;
        std::lock_guard<std::mutex> lock(g_attr_mu);
        g_row_scan_occ.emplace_back(key, smem, per_sm);
    }
    if (per_sm < 1) per_sm = 1;
    int64_t ctas = static_cast<int64_t>(num_sms) * per_sm;
    const int64_t need = (rows + kScanWarpsPerCta - 1) / kScanWarpsPerCta;
    if (ctas > need) ctas = need;
    // The speculative threshold pays off over several rows per warp; with
    // few rows a failed guess (a second read of the row) only adds to the tail.
    int speculate = (max_C > 32 && rows >= 4 * ctas * kScanWarpsPerCta) ? 1 : 0;
    if (speculate_mode > 0 && max_C > 32) speculate = 1;
    const dim3 grid(static_cast<unsigned>(ctas));
    if (k16) row_scan_kernel<true><<<grid, threads, smem, stream>>>(p, capw, speculate);
    else row_scan_kernel<false><<<grid, threads, smem, stream>>>(p, capw, speculate);
    return counted(cudaGetLastError());
}

// DBS_LIST_MERGE=0 turns the compact merge off (read once, for measurements).
static bool list_merge_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("DBS_LIST_MERGE");
        return !(v && std::atoi(v) == 0);
    }();
    return on;
}

static size_t merge_rank_smem(int ring, int max_K, int max_C, int max_N, int tab_n) {
    size_t b = static_cast<size_t>(2) * tab_n * sizeof(float);              // length-penalty tables
    b += static_cast<size_t>(ring) * max_K * max_C * sizeof(uint64_t);      // ring lists
    b += static_cast<size_t>(4) * max_N * sizeof(uint64_t);                 // top-N hi/lo, double buffered
    b += static_cast<size_t>(2) * (max_N + kRescanChunk) * sizeof(uint64_t); // rescan staging
    b += static_cast<size_t>(2) * max_K * sizeof(uint64_t);                 // carry keys
    b += static_cast<size_t>(ring) * max_K * (sizeof(float) + sizeof(int)); // ring bounds / counts
    b += static_cast<size_t>(2) * max_K * (2 * sizeof(float) + 2 * sizeof(int));
    return b;
}

// Shared memory the ranking merge may take; beyond it the sort merge runs.
constexpr size_t kMergeRankSmemBudget = 200 * 1024;

bool compact_merge_applies(int max_K, int max_C, int max_ext, int max_N, bool need_sequences,
                           bool first_row_apart) {
    const int64_t M = static_cast<int64_t>(max_K) * max_C;
    if (!need_sequences && !first_row_apart && M <= 256) return false;   // the ranking merge
    return !need_sequences && M + max_ext <= kListMergeMaxCandidates && max_N <= kListMergeThreads &&
           list_merge_enabled();
}

cudaError_t launch_step_merge(const DecodeParams& p, int max_K, int max_C, int max_T, int max_N,
                              bool need_sequences, cudaStream_t stream, int max_threads, int max_ext) {
    // (the ranking merge reads every row as one list of at most C entries)
    if (!need_sequences && !p.first_row_apart && static_cast<int64_t>(max_K) * max_C <= 256) {
        const int tab_n = (p.Lmax + 1 <= 4096) ? p.Lmax + 1 : 0;
        int ring = max_T < kMergeRingMax ? max_T : kMergeRingMax;
        if (ring < 2) ring = 2;
        while (ring > 2 && merge_rank_smem(ring, max_K, max_C, max_N, tab_n) > kMergeRankSmemBudget) --ring;
        const size_t smem = merge_rank_smem(ring, max_K, max_C, max_N, tab_n);
        if (smem <= kMergeRankSmemBudget) {
            int lanes = 1;
            while (lanes < max_K && lanes < 32) lanes <<= 1;
            const int64_t work = (static_cast<int64_t>(max_K) * max_C + max_K) * lanes;
            // at most 768 threads (48K registers): a CTA always fits beside one
            // 512-thread zero-fill block on the same SM
            constexpr int kCap = 768;
            int threads = static_cast<int>(work < kCap ? work : kCap);
            threads = ((threads + 31) / 32) * 32;
            if (threads < 64) threads = 64;
            cudaError_t err = ensure_dynamic_smem(reinterpret_cast<const void*>(step_merge_rank_kernel), smem);
            if (err != cudaSuccess) return err;
            step_merge_rank_kernel<<<p.B, threads, smem, stream>>>(p, ring, max_K, max_C, max_N, tab_n);
            return counted(cudaGetLastError());
        }
    }
    const int M = max_K * max_C;
    if (!need_sequences && M + max_ext <= kListMergeMaxCandidates && max_N <= kListMergeThreads &&
        list_merge_enabled()) {
        // compact merge: candidate keys in registers, radix select, ranking by counting
        constexpr int nt = kListMergeThreads;
        const int sel_cap = list_merge_sel_cap(max_N, nt);
        // the next step's lists are prefetched into shared memory
        const int pf_cap = (M + max_ext + 1) & ~1;
        const size_t smem = align16(list_merge_smem(nt, sel_cap, max_K)) + merge_prefetch_bytes(pf_cap, max_K);
        const int per = M + max_ext <= nt * 4 ? 4 : (M + max_ext <= nt * 5 ? 5 : 8);
        const void* fn = per == 4 ? reinterpret_cast<const void*>(list_merge_kernel<nt, 4>)
                                  : (per == 5 ? reinterpret_cast<const void*>(list_merge_kernel<nt, 5>)
                                              : reinterpret_cast<const void*>(list_merge_kernel<nt, 8>));
        cudaError_t err = ensure_dynamic_smem(fn, smem);
        if (err != cudaSuccess) return err;
        if (per == 4) list_merge_kernel<nt, 4><<<p.B, nt, smem, stream>>>(p, max_K, sel_cap, pf_cap);
        else if (per == 5) list_merge_kernel<nt, 5><<<p.B, nt, smem, stream>>>(p, max_K, sel_cap, pf_cap);
        else list_merge_kernel<nt, 8><<<p.B, nt, smem, stream>>>(p, max_K, sel_cap, pf_cap);
        return counted(cudaGetLastError());
    }
    int cand_cap = M;
    if (cand_cap < max_N + 2048) cand_cap = max_N + 2048;
    const int sel_cap = max_N + 2048;
    // prefix filters of the sequence constraints: two buffers of K filters
    const int bloom_log2 = !need_sequences ? 0 : (max_K <= 32 ? 11 : (max_K <= 64 ? 10 : 0));
    const int bloom_words = bloom_log2 ? 1 << (bloom_log2 - 5) : 0;
    size_t smem = static_cast<size_t>(cand_cap) * 2 * sizeof(uint64_t) +
                  static_cast<size_t>(max_K) * 3 * sizeof(float) +
                  static_cast<size_t>(max_K) * 7 * sizeof(int) + 64 +
                  16 + static_cast<size_t>(sel_cap) * 2 * sizeof(uint64_t) +
                  static_cast<size_t>(2) * max_K * bloom_words * sizeof(uint32_t);
    // prefixes (two buffers) and n-gram sets in shared memory when they fit
    const size_t seq_bytes = static_cast<size_t>(3) * max_K * max_T * sizeof(int32_t);
    const int seq_smem = (need_sequences && smem + seq_bytes <= 200 * 1024) ? 1 : 0;
    if (seq_smem) smem += seq_bytes;
    // about two candidates per thread (the run merges of a step are bound by
    // shared-memory latency, so more warps help)
    int threads = 64;
    while (threads < kMergeThreads && threads * 2 <= M) threads <<= 1;
    if (threads < 128 && max_K > 64) threads = 128;
    // More examples than SMs: 256-thread CTAs, two per SM (a 512-thread CTA
    // holds an SM's registers), so the examples run in one wave, not two.
    int dev = 0, sms = 0;
    cudaError_t aerr = cudaGetDevice(&dev);
    if (aerr == cudaSuccess) aerr = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (aerr != cudaSuccess) return aerr;
    if (p.B > sms && threads > 256) threads = 256;
    if (max_threads > 0 && threads > max_threads) threads = max_threads;
    const bool runs = !need_sequences && M <= 1024;
    const void* fn = runs ? reinterpret_cast<const void*>(step_merge_kernel<true>)
                          : reinterpret_cast<const void*>(step_merge_kernel<false>);
    cudaError_t err = ensure_dynamic_smem(fn, smem);
    if (err != cudaSuccess) return err;
    if (runs) step_merge_kernel<true><<<p.B, threads, smem, stream>>>(p, cand_cap, max_T, max_K, sel_cap, bloom_log2, seq_smem);
    else step_merge_kernel<false><<<p.B, threads, smem, stream>>>(p, cand_cap, max_T, max_K, sel_cap, bloom_log2, seq_smem);
    return counted(cudaGetLastError());
}

cudaError_t launch_fused_decode(const DecodeParams& p, int max_K, int max_C, int max_ext, int max_N,
                                int merge_ctas, unsigned int* step_done, int num_sms, cudaStream_t stream) {
    const int M = max_K * max_C + max_ext;
    if (M > 8 * kFusedThreads || max_N > kFusedThreads || merge_ctas < 1) return cudaErrorNotSupported;
    const int capw = row_scan_capw(max_C + max_ext);
    const int sel_cap = list_merge_sel_cap(max_N, kFusedThreads);
    size_t smem = static_cast<size_t>(kFusedThreads / 32) * row_scan_warp_bytes(capw, false);
    const int per = M <= kFusedThreads * 4 ? 4 : (M <= kFusedThreads * 5 ? 5 : 8);
    // the dynamic shared memory a CTA can have beside the kernel's static arrays
    size_t smem_max = 0;
    {
        const void* f = per == 4 ? reinterpret_cast<const void*>(fused_decode_kernel<4>)
                                 : (per == 5 ? reinterpret_cast<const void*>(fused_decode_kernel<5>)
                                             : reinterpret_cast<const void*>(fused_decode_kernel<8>));
        cudaFuncAttributes fa{};
        int dev = 0, optin = 0;
        cudaError_t e = cudaFuncGetAttributes(&fa, f);
        if (e == cudaSuccess) e = cudaGetDevice(&dev);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (e != cudaSuccess) return e;
        smem_max = static_cast<size_t>(optin) > fa.sharedSizeBytes ? static_cast<size_t>(optin) - fa.sharedSizeBytes : 0;
    }
    // a merge CTA with several examples keeps their beams after its arrays,
    // then each example's prefetch block (left out when it does not fit)
    const int per_cta = (p.B + merge_ctas - 1) / merge_ctas;
    const size_t mbase = align16(list_merge_smem(kFusedThreads, sel_cap, max_K)) +
                         align16(static_cast<size_t>(per_cta > 1 ? per_cta : 0) * 3 * max_K * sizeof(float));
    int pf_cap = (M + 1) & ~1;
    if (mbase + static_cast<size_t>(per_cta) * merge_prefetch_bytes(pf_cap, max_K) > smem_max) pf_cap = 0;
    const size_t msmem = mbase + (pf_cap ? static_cast<size_t>(per_cta) * merge_prefetch_bytes(pf_cap, max_K) : 0);
    if (msmem > smem) smem = msmem;
    if (smem > smem_max) return cudaErrorNotSupported;
    const void* fn = per == 4 ? reinterpret_cast<const void*>(fused_decode_kernel<4>)
                              : (per == 5 ? reinterpret_cast<const void*>(fused_decode_kernel<5>)
                                          : reinterpret_cast<const void*>(fused_decode_kernel<8>));
    cudaError_t err = ensure_dynamic_smem(fn, smem);
    if (err != cudaSuccess) return err;
    int per_sm = 0;
    err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kFusedThreads, smem);
    if (err != cudaSuccess) return err;
    const int grid = per_sm * num_sms;
    if (per_sm < 1 || grid <= merge_ctas) return cudaErrorNotSupported;
    DecodeParams pp = p;
    int a_capw = capw, a_seq = max_K, a_sel = sel_cap, a_m = merge_ctas, a_pf = pf_cap;
    unsigned int* a_done = step_done;
    void* args[] = {&pp, &a_capw, &a_seq, &a_sel, &a_m, &a_done, &a_pf};
    err = cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(kFusedThreads), args, smem, stream);
    return counted(err);
}

cudaError_t launch_weights(const DecodeParams& p, int max_T, int max_K, int max_P, cudaStream_t stream) {
    (void)max_K;
    const int64_t warps = static_cast<int64_t>(p.B) * max_T;
    const int threads = 256;
    const int64_t blocks = (warps * 32 + threads - 1) / threads;
    cudaError_t err = cudaSuccess;
    if (max_P <= 32) err = prefer_shared(reinterpret_cast<const void*>(weights_kernel<32>));
    else if (max_P <= 128) err = prefer_shared(reinterpret_cast<const void*>(weights_kernel<128>));
    else if (max_P <= 512) err = prefer_shared(reinterpret_cast<const void*>(weights_kernel<512>));
    else if (max_P <= 1024) err = prefer_shared(reinterpret_cast<const void*>(weights_kernel<1024>));
    if (err != cudaSuccess) return err;
    if (max_P <= 32) weights_kernel<32><<<blocks, threads, 0, stream>>>(p, max_T);
    else if (max_P <= 128) weights_kernel<128><<<blocks, threads, 0, stream>>>(p, max_T);
    else if (max_P <= 512) weights_kernel<512><<<blocks, threads, 0, stream>>>(p, max_T);
    else if (max_P <= 1024) weights_kernel<1024><<<blocks, threads, 0, stream>>>(p, max_T);
    else return cudaErrorInvalidValue;
    return counted(cudaGetLastError());
}

static size_t backward_sweep_smem(int max_T, int max_K, int max_P, bool with_pool) {
    size_t b = static_cast<size_t>(max_T) * max_K * (sizeof(float) + 2 * sizeof(int));
    b += static_cast<size_t>(max_T) * (2 * sizeof(float) + sizeof(int));
    if (with_pool) b += static_cast<size_t>(max_T) * max_P * (sizeof(int) + sizeof(float));
    return b;
}
constexpr size_t kBackwardSweepSmemBudget = 96 * 1024;

static size_t backward_smem_bytes(int max_K, int max_P) {
    return static_cast<size_t>(max_K) * 3 * sizeof(float) + static_cast<size_t>(max_P) * sizeof(float) +
           static_cast<size_t>(max_K + max_P) * sizeof(int) + 16 +
           static_cast<size_t>(max_K + max_P) * (sizeof(int64_t) + sizeof(float));
}

cudaError_t launch_backward(const BackwardParams& p, int max_K, int max_P, bool sparse, cudaStream_t stream) {
    // the sweep: dense output, or sparse output without a relaxed-pool gradient
    if (max_K <= 32 && (sparse ? p.grad_relaxed == nullptr : p.grad_dense != nullptr)) {
        const bool with_pool = !sparse && p.grad_relaxed != nullptr;
        const size_t smem = backward_sweep_smem(p.max_T, max_K, max_P, with_pool);
        if (smem <= kBackwardSweepSmemBudget) {
            cudaError_t err = ensure_dynamic_smem(reinterpret_cast<const void*>(backward_sweep_kernel), smem);
            if (err != cudaSuccess) return err;
            backward_sweep_kernel<<<p.B, 256, smem, stream>>>(p, p.max_T, max_K, max_P, with_pool ? 1 : 0,
                                                              sparse ? 1 : 0);
            return counted(cudaGetLastError());
        }
    }
    const size_t smem = backward_smem_bytes(max_K, max_P);
    cudaError_t err = ensure_dynamic_smem(reinterpret_cast<const void*>(backward_kernel), smem);
    if (err != cudaSuccess) return err;
    int threads = 128;
    if (max_P > 512) threads = 256;
    backward_kernel<<<p.B, threads, smem, stream>>>(p, sparse ? 1 : 0, max_K, max_P);
    return counted(cudaGetLastError());
}

cudaError_t launch_fill_zero_bulk(float* dst, int64_t count, int num_sms, cudaStream_t stream) {
    if (count <= 0) return cudaSuccess;
    cudaError_t err = ensure_dynamic_smem(reinterpret_cast<const void*>(fill_zero_bulk_kernel), kFillTileBytes);
    if (err != cudaSuccess) return err;
    const int64_t tiles = (count * 4 + kFillTileBytes - 1) / kFillTileBytes;
    int64_t blocks = num_sms;
    if (blocks > tiles) blocks = tiles;
    if (blocks < 1) blocks = 1;
    fill_zero_bulk_kernel<<<static_cast<unsigned>(blocks), 32, kFillTileBytes, stream>>>(dst, count);
    return counted(cudaGetLastError());
}

cudaError_t launch_fill_zero(float* dst, int64_t count, int num_sms, cudaStream_t stream, int blocks_per_sm) {
    if (count <= 0) return cudaSuccess;
    const int threads = 512;
    int64_t blocks = (count / 4 + threads - 1) / threads;
    const int64_t max_blocks = static_cast<int64_t>(num_sms) * blocks_per_sm;
    if (blocks > max_blocks) blocks = max_blocks;
    if (blocks < 1) blocks = 1;
    cudaError_t err = prefer_shared(reinterpret_cast<const void*>(fill_zero_kernel));
    if (err != cudaSuccess) return err;
    fill_zero_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(dst, count);
    return counted(cudaGetLastError());
}


// ---------------------------------------------------------------------------
// Sparse backward that allocates nothing (dbs_device_backward_sparse_noalloc).
//
// Callers that may not allocate device memory on their call path (code that
// runs while a framework's caching allocator owns the device, inside a
// capture or replay region it manages, or in a real-time loop where
// cudaMalloc's implicit synchronisation is not acceptable) still need the
// sparse backward. Its only scratch, the per-(example, step) entry counts
// used to compact the sparse segments, lives in the file-scope array below;
// the example descriptors of the uniform batch are computed in the kernel and
// the 1/gnmt table travels in the kernel parameters. Every scratch slot is
// written before it is read, so nothing has to start at zero.
//
// Limits: batch_size * steps <= kNoAllocMaxStepCounts (1 MiB of scratch),
// steps <= kNoAllocMaxSteps (the parameter table), beam + pool <= 4096.
// There is one scratch array per device, so calls on one device must not
// overlap in time (on different streams they would race on it); calls in a
// row on one stream are ordered and safe.
// ---------------------------------------------------------------------------
static __device__ __align__(256) int32_t g_noalloc_step_counts[kNoAllocMaxStepCounts];

struct NoAllocPenalty {
    float inv_pen[kNoAllocMaxSteps + 2];   // 1 / gnmt(l), l = 0 .. steps + 1
};

__global__ void backward_noalloc_kernel(BackwardParams p, int T, int K, int P, NoAllocPenalty tab,
                                        int32_t* scratch) {
    const int e = blockIdx.x;
    ExampleDesc d{};
    d.T = T;
    d.K = K;
    d.P = P;
    d.sel_offset = static_cast<int64_t>(e) * T * K;
    d.pool_offset = static_cast<int64_t>(e) * T * P;
    d.final_offset = static_cast<int64_t>(e) * K;
    d.sparse_offset = static_cast<int64_t>(e) * T * (K + P);
    d.sel_stride = K;
    d.pool_stride = P;
    d.sel_t_stride = K;
    d.pool_t_stride = P;
    backward_example(p, d, e, tab.inv_pen, scratch, 1, K, P);
}

// Scratch address per device, looked up once with that device current.
static std::mutex g_noalloc_mu;
static std::vector<int32_t*> g_noalloc_ptr;

static cudaError_t noalloc_scratch(int32_t** out) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (dev >= static_cast<int>(g_noalloc_ptr.size())) g_noalloc_ptr.resize(dev + 1, nullptr);
    if (!g_noalloc_ptr[dev]) {
        void* ptr = nullptr;
        err = cudaGetSymbolAddress(&ptr, g_noalloc_step_counts);
        if (err != cudaSuccess) return err;
        g_noalloc_ptr[dev] = static_cast<int32_t*>(ptr);
    }
    *out = g_noalloc_ptr[dev];
    return cudaSuccess;
}

cudaError_t noalloc_prepare() {
    int32_t* ptr = nullptr;
    cudaError_t err = noalloc_scratch(&ptr);
    if (err != cudaSuccess) return err;
    return ensure_dynamic_smem(reinterpret_cast<const void*>(backward_noalloc_kernel),
                               backward_smem_bytes(kNoAllocMaxBeamPlusPool, 0));
}

cudaError_t launch_backward_noalloc(const BackwardParams& p, int T, int K, int P, const float* inv_pen_host,
                                    cudaStream_t stream) {
    if (T < 1 || T > kNoAllocMaxSteps || K < 1 || P < K || K + P > kNoAllocMaxBeamPlusPool ||
        static_cast<int64_t>(p.B) * T > kNoAllocMaxStepCounts)
        return cudaErrorInvalidValue;
    int32_t* scratch = nullptr;
    cudaError_t err = noalloc_prepare();
    if (err != cudaSuccess) return err;
    err = noalloc_scratch(&scratch);
    if (err != cudaSuccess) return err;
    NoAllocPenalty tab{};
    for (int l = 0; l < T + 2; ++l) tab.inv_pen[l] = inv_pen_host[l];
    BackwardParams q = p;
    q.desc = nullptr;
    q.inv_pen = nullptr;
    q.step_counts = scratch;
    q.max_T = T;
    const size_t smem = backward_smem_bytes(K, P);
    const int threads = P > 512 ? 256 : 128;
    backward_noalloc_kernel<<<p.B, threads, smem, stream>>>(q, T, K, P, tab, scratch);
    return counted(cudaGetLastError());
}

}  // namespace dbs_dev
