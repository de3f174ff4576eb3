// st_gemm_group.cuh -- the persistent grouped TF32 GEMM: several dependent
// GEMMs (the six of an MLP layer's forward + backward) in one launch.
//
// Included by st_gemm.cu inside its anonymous namespace, after GemmArgs, the
// epilogue helpers and epilogue_tma.
//
// Why.  At the tiny shapes of the reference's models (d_model 32-256) a
// single GEMM is a few microseconds of work; launching six of them, each with
// its own prologue, pipeline fill and epilogue drain, and its own split-k
// reduction, costs several times the work.  Here two CTAs per SM each run a loop
// over tasks (one output tile, or one split of one) taken from a global ticket
// counter, so tiles of the next GEMM start the moment their inputs exist, and
// the epilogue of one task overlaps the main loop of the next (two TMEM
// accumulators).  Tickets are handed out in order and a task only depends on
// tasks with lower tickets, so the lowest unfinished task always belongs to a
// running CTA: the scheme cannot deadlock, whatever else shares the GPU.
//
// Roles (6 warps): warp 0 takes tickets, waits for the GEMMs a task reads and
// streams its operands by TMA; warp 1 issues the tcgen05 MMAs into one of two
// TMEM accumulators; warps 2-5 drain an accumulator through the epilogue and
// TMA stores.  A split task stores a raw partial and counts itself in a
// per-tile counter; reduction tasks (row bands of the tile, later tickets)
// wait for that count, sum the partials in split order and apply the
// epilogue -- the same bits as st_gemm's split-k reduction.
// Dependencies are per GEMM: a counter of finished output tiles, written with
// release semantics after the tile's stores have completed, read with acquire
// semantics (then a proxy fence, since the reads are TMA loads).

constexpr int GRP_MAX = 8;        // GEMMs per group
constexpr int GRP_STAGES = 2;     // operand ring depth (two CTAs per SM)
constexpr int GRP_BNMAX = 128;    // widest tile; TMEM holds two accumulators of this width
constexpr int GRP_STAGE_BYTES = (BM + GRP_BNMAX) * BK * 4;
constexpr int GRP_RING = GRP_STAGES * GRP_STAGE_BYTES;
constexpr int GRP_EPI_BYTES = 4 * 8192;  // per epilogue warp: two 4 KB store boxes
constexpr int GRP_SMEM = GRP_RING + GRP_EPI_BYTES + 512 + 1024;
constexpr int GRP_THREADS = 192;

struct GroupMaps {
    CUtensorMap tmA, tmB, tmC, tmP;  // operands, output, split partials [splits][M][N]
};

// The scalar part of a GEMM of the group; the kernel copies these to shared
// memory once (reading a kernel parameter at a computed index goes through
// the constant cache, far slower than shared memory).
struct GroupGemm {
    GemmArgs g;                      // shape and epilogue (batch 1)
    int a_mn, b_mn, bn;
    int m_tiles, n_tiles, splits, kb_per_split;
    int red_parts;    // split GEMMs: reduction tasks per tile (row bands of BM / red_parts)
    int need;         // finished units that complete the GEMM: tiles, or tiles * red_parts
    int task_begin;   // first ticket of this GEMM: tiles * splits MMA tasks, then tiles * red_parts reductions
    int tile_begin;   // first per-tile split counter
    uint32_t after;   // bit j: reads the output of GEMM j
};

struct GroupPlan {
    GroupMaps maps[GRP_MAX];
    GroupGemm gemm[GRP_MAX];
    int count, tasks;
    // [0] ticket, [1] abort, [2] CTAs finished, [3..3+GRP_MAX) finished units per GEMM, then per-tile
    // split counters.  All zero between launches: the last CTA to finish resets them.
    unsigned int *ctl;
    int ctl_words;
    int *status;
};

constexpr int CTL_TICKET = 0, CTL_ABORT = 1, CTL_EXIT = 2, CTL_DONE = 3, CTL_TILES = 3 + GRP_MAX;

__device__ __forceinline__ unsigned int ld_acquire(const unsigned int *p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add(unsigned int *p, unsigned int v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// orders this thread's earlier generic-proxy accesses with its later
// async-proxy (TMA) accesses of global memory, and vice versa
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void epi_bar() {  // the four epilogue warps
    asm volatile("bar.sync 1, 128;" ::: "memory");
}
// Barrier of the four epilogue warps that also ANDs a flag over them, so that
// they always take the same branch (a warp leaving alone would strand the
// others in the next barrier).
__device__ __forceinline__ bool epi_all(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, 1, 128, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(v))
        : "memory");
    return r != 0;
}

// Which GEMM a ticket belongs to.
__device__ __forceinline__ int group_of(const GroupGemm *gs, int count, int t) {
    int gi = 0;
#pragma unroll 1
    for (int j = 1; j < count; j++)
        if (t >= gs[j].task_begin) gi = j;
    return gi;
}

// Waits until every GEMM in `after` has finished all its tiles (bounded;
// raises the plan's abort flag on expiry).  Returns false on abort.
__device__ bool wait_after(const GroupPlan &p, const GroupGemm *gs, uint32_t after) {
    const uint64_t t0 = st::globaltimer();
#pragma unroll 1
    for (int j = 0; j < p.count; j++) {
        if (!(after & (1u << j))) continue;
        const unsigned int need = static_cast<unsigned int>(gs[j].need);
#pragma unroll 1
        for (uint32_t i = 0;; ++i) {
            if (ld_acquire(p.ctl + CTL_DONE + j) >= need) break;
            if (ld_acquire(p.ctl + CTL_ABORT)) return false;
            __nanosleep(200);
            if ((i & 15u) == 0 && st::globaltimer() - t0 > st::WAIT_LIMIT_NS) {
                st::set_status(p.status, st::DEV_TIMEOUT_FULL);
                atomicExch(p.ctl + CTL_ABORT, 1u);
                return false;
            }
        }
    }
    if (after) fence_proxy_async_global();
    return true;
}

// Reduction task: rows [r0, r1) x columns [n0, n0 + bn) of a split GEMM's
// output = the split partials summed in split order, then the epilogue.  The
// 128 epilogue threads take float4 groups row-major (coalesced per split);
// each keeps 16 partial loads in flight.
__device__ void group_reduce(const GroupGemm &G, int r0, int r1, int n0, int tid) {
    const GemmArgs &g = G.g;
    const int groups = G.bn / 4;
    const int64_t mn = static_cast<int64_t>(g.M) * g.N;
    r1 = min(r1, g.M);
#pragma unroll 1
    for (int e = tid; e < (r1 - r0) * groups; e += 128) {
        const int row = r0 + e / groups, col = n0 + 4 * (e % groups);
        if (col >= g.N) continue;
        const float *p = g.partial + static_cast<int64_t>(row) * g.N + col;
        float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 1
        for (int sp0 = 0; sp0 < G.splits; sp0 += 16) {
            float4 v[16];
#pragma unroll
            for (int j = 0; j < 16; j++)
                v[j] = (sp0 + j < G.splits) ? __ldcg(reinterpret_cast<const float4 *>(p + (sp0 + j) * mn))
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int j = 0; j < 16; j++) {
                if (sp0 + j >= G.splits) break;
                s[0] = __fadd_rn(s[0], v[j].x);
                s[1] = __fadd_rn(s[1], v[j].y);
                s[2] = __fadd_rn(s[2], v[j].z);
                s[3] = __fadd_rn(s[3], v[j].w);
            }
        }
        const int64_t oi = out_index(g, 0, row, col);
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; j++) o[j] = epilogue(g, 0, oi + j, col + j, s[j]);
        *reinterpret_cast<float4 *>(g.c + oi) = make_float4(o[0], o[1], o[2], o[3]);
    }
}

// The task a ticket names: GEMM, tile origin, and either a split (an MMA
// task) or a row band (a reduction task of a split GEMM).
struct GroupTask {
    int gi, m0, n0, tile;
    int split;  // MMA task: the split; reduction task: -1
    int part;   // reduction task: the row band
};
__device__ __forceinline__ GroupTask decode_task(const GroupGemm *gs, int count, int t) {
    GroupTask k;
    k.gi = group_of(gs, count, t);
    const GroupGemm &G = gs[k.gi];
    const int tiles = G.m_tiles * G.n_tiles;
    int r = t - G.task_begin;
    if (r < tiles * G.splits) {
        k.split = r % G.splits;
        k.tile = r / G.splits;
        k.part = 0;
    } else {
        r -= tiles * G.splits;
        k.split = -1;
        k.tile = r / G.red_parts;
        k.part = r % G.red_parts;
    }
    k.m0 = (k.tile / G.n_tiles) * BM;
    k.n0 = (k.tile % G.n_tiles) * G.bn;
    return k;
}

// Spins (bounded) until *ctr >= need; false on abort or expiry.
__device__ bool wait_count(const GroupPlan &p, const unsigned int *ctr, unsigned int need) {
    const uint64_t t0 = st::globaltimer();
#pragma unroll 1
    for (uint32_t i = 0;; ++i) {
        if (ld_acquire(ctr) >= need) return true;
        if (ld_acquire(p.ctl + CTL_ABORT)) return false;
        __nanosleep(100);
        if ((i & 15u) == 0 && st::globaltimer() - t0 > st::WAIT_LIMIT_NS) {
            st::set_status(p.status, st::DEV_TIMEOUT_FULL);
            atomicExch(p.ctl + CTL_ABORT, 1u);
            return false;
        }
    }
}

__global__ void __launch_bounds__(GRP_THREADS, 2) k_gemm_group(const __grid_constant__ GroupPlan p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *epi_smem = smem + GRP_RING;
    uint64_t *full = reinterpret_cast<uint64_t *>(epi_smem + GRP_EPI_BYTES);
    uint64_t *empty = full + GRP_STAGES;
    uint64_t *acc_full = empty + GRP_STAGES;  // [2]
    uint64_t *acc_empty = acc_full + 2;       // [2]
    uint64_t *sched_full = acc_empty + 2;     // [2]
    uint64_t *sched_empty = sched_full + 2;   // [2]
    int *sched_task = reinterpret_cast<int *>(sched_empty + 2);  // [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sched_task + 2);

    __shared__ GroupGemm gs[GRP_MAX];
    for (int i = threadIdx.x; i < p.count * static_cast<int>(sizeof(GroupGemm) / 4); i += blockDim.x)
        reinterpret_cast<uint32_t *>(gs)[i] = reinterpret_cast<const uint32_t *>(p.gemm)[i];
    const int count = p.count;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < GRP_STAGES; s++) {
            st::mbar_init(&full[s], 1);
            st::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            st::mbar_init(&acc_full[b], 1);
            st::mbar_init(&acc_empty[b], 4);
            st::mbar_init(&sched_full[b], 1);
            st::mbar_init(&sched_empty[b], 5);
        }
        st::fence_mbar_init();
    }
    if (warp == 1) {
        st::tmem_alloc(tmem_slot, 2 * GRP_BNMAX);
        st::tmem_relinquish();
    } else if (warp == 0) {
        for (int j = lane; j < 2 * p.count; j += 32)
            st::tma_prefetch_desc(j & 1 ? &p.maps[j >> 1].tmB : &p.maps[j >> 1].tmA);
    } else if (warp == 2) {
        for (int j = lane; j < p.count; j += 32) {
            st::tma_prefetch_desc(&p.maps[j].tmC);
            if (p.gemm[j].splits > 1) st::tma_prefetch_desc(&p.maps[j].tmP);
        }
    }
    st::tc_fence_before();
    __syncthreads();
    st::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    st::grid_dep_wait();

    if (warp == 0) {
        if (lane == 0) {  // ticket taker and TMA producer
            int it = 0;   // k blocks issued so far (ring position)
#pragma unroll 1
            for (int j = 0;; ++j) {
                const int slot = j & 1;
                if (j >= 2 && !st::mbar_wait(&sched_empty[slot], ((j >> 1) - 1) & 1, p.status, st::DEV_TIMEOUT_EMPTY))
                    break;
                int t = static_cast<int>(atomicAdd(p.ctl + CTL_TICKET, 1u));
                if (t >= p.tasks || ld_acquire(p.ctl + CTL_ABORT)) t = -1;
                sched_task[slot] = t;
                st::mbar_arrive(&sched_full[slot]);
                if (t < 0) break;
                const GroupTask k = decode_task(gs, count, t);
                if (k.split < 0) continue;  // a reduction: no operands
                const GroupGemm &G = gs[k.gi];
                const GroupMaps &MP = p.maps[k.gi];
                if (!wait_after(p, gs, G.after)) break;  // abort: the consumers of this task time out
                const int kb_total = (G.g.K + BK - 1) / BK;
                const int kb0 = k.split * G.kb_per_split;
                const int nkb = max(0, min(kb_total, kb0 + G.kb_per_split) - kb0);
                const uint32_t bytes = static_cast<uint32_t>((BM + G.bn) * BK * 4);
                bool ok = true;
#pragma unroll 1
                for (int i = 0; i < nkb; i++, it++) {
                    const int s = it % GRP_STAGES;
                    if (it >= GRP_STAGES &&
                        !st::mbar_wait(&empty[s], ((it / GRP_STAGES) - 1) & 1, p.status, st::DEV_TIMEOUT_EMPTY)) {
                        ok = false;
                        break;
                    }
                    st::mbar_arrive_expect_tx(&full[s], bytes);
                    const int kc = (kb0 + i) * BK;
                    uint8_t *sa = smem + s * GRP_STAGE_BYTES;
                    uint8_t *sb = sa + BM * BK * 4;
                    if (!G.a_mn) {
                        st::tma_load_4d(sa, &MP.tmA, &full[s], kc, k.m0, 0, 0);
                    } else {
#pragma unroll
                        for (int c = 0; c < BM / 32; c++) st::tma_load_4d(sa + c * 4096, &MP.tmA, &full[s], k.m0 + 32 * c, kc, 0, 0);
                    }
                    if (!G.b_mn) {
                        st::tma_load_4d(sb, &MP.tmB, &full[s], kc, k.n0, 0, 0);
                    } else {
#pragma unroll 1
                        for (int c = 0; c < G.bn / 32; c++) st::tma_load_4d(sb + c * 4096, &MP.tmB, &full[s], k.n0 + 32 * c, kc, 0, 0);
                    }
                }
                if (!ok) break;
            }
            // the CTA may not exit with loads still landing in its shared memory
            for (int s = 0; s < GRP_STAGES && s < it; s++) {
                const int last = it - 1 - ((it - 1 - s) % GRP_STAGES);  // last k block issued into stage s
                (void)st::mbar_wait(&full[last % GRP_STAGES], (last / GRP_STAGES) & 1, p.status, st::DEV_TIMEOUT_FULL);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            int it = 0, mj = 0;  // ring position; MMA tasks so far (accumulator = mj & 1)
#pragma unroll 1
            for (int j = 0;; ++j) {
                const int slot = j & 1;
                if (!st::mbar_wait(&sched_full[slot], (j >> 1) & 1, p.status, st::DEV_TIMEOUT_FULL)) break;
                const int t = sched_task[slot];
                st::mbar_arrive(&sched_empty[slot]);
                if (t < 0) break;
                const GroupTask k = decode_task(gs, count, t);
                if (k.split < 0) continue;
                const GroupGemm &G = gs[k.gi];
                const int buf = mj & 1;
                const int kb_total = (G.g.K + BK - 1) / BK;
                const int kb0 = k.split * G.kb_per_split;
                const int nkb = max(0, min(kb_total, kb0 + G.kb_per_split) - kb0);
                if (mj >= 2 && !st::mbar_wait(&acc_empty[buf], ((mj >> 1) - 1) & 1, p.status, st::DEV_TIMEOUT_ACC))
                    break;
                ++mj;
                st::tc_fence_after();
                const uint32_t d = tmem + static_cast<uint32_t>(buf * GRP_BNMAX);
                const uint32_t idesc = (G.bn == 128 ? st::idesc_make(1, 2, false, false, BM, 128)
                                                    : st::idesc_make(1, 2, false, false, BM, 64)) |
                                       (G.a_mn ? (1u << 15) : 0u) | (G.b_mn ? (1u << 16) : 0u);
                bool ok = true;
#pragma unroll 1
                for (int i = 0; i < nkb; i++, it++) {
                    const int s = it % GRP_STAGES;
                    if (!st::mbar_wait(&full[s], (it / GRP_STAGES) & 1, p.status, st::DEV_TIMEOUT_FULL)) {
                        ok = false;
                        break;
                    }
                    st::tc_fence_after();
                    const uint32_t sa = st::smem_u32(smem + s * GRP_STAGE_BYTES);
                    const uint32_t sb = sa + BM * BK * 4;
#pragma unroll
                    for (int kk = 0; kk < BK / 8; kk++) {
                        const uint64_t ad = G.a_mn ? st::sdesc_make(sa + kk * 1024, 4096, 512, st::LAYOUT_SW128_BASE32B)
                                                   : st::sdesc_sw128(sa + kk * 32, 16, 1024);
                        const uint64_t bd = G.b_mn ? st::sdesc_make(sb + kk * 1024, 4096, 512, st::LAYOUT_SW128_BASE32B)
                                                   : st::sdesc_sw128(sb + kk * 32, 16, 1024);
                        st::umma_tf32(d, ad, bd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
                    }
                    st::umma_commit(&empty[s]);
                }
                if (!ok) break;
                st::umma_commit(&acc_full[buf]);
            }
        }
    } else {  // warps 2..5: epilogue and reductions; warp w drains TMEM lanes 32*(w%4) ..
        const int q = warp & 3, tid = threadIdx.x - 64;
        uint8_t *stage = epi_smem + q * 8192;
        int mj = 0;  // MMA tasks drained so far (accumulator = mj & 1)
#pragma unroll 1
        for (int j = 0;; ++j) {
            const int slot = j & 1;
            bool ok = st::mbar_wait(&sched_full[slot], (j >> 1) & 1, p.status, st::DEV_TIMEOUT_FULL);
            const int t = ok ? sched_task[slot] : -1;
            __syncwarp();
            if (ok && lane == 0) st::mbar_arrive(&sched_empty[slot]);
            GroupTask k{};
            if (t >= 0) k = decode_task(gs, count, t);
            const bool mma_task = t >= 0 && k.split >= 0;
            const int buf = mj & 1;
            if (mma_task) {
                ok = ok && st::mbar_wait(&acc_full[buf], (mj >> 1) & 1, p.status, st::DEV_TIMEOUT_ACC);
            } else if (t >= 0 && tid == 0) {  // a reduction waits until every split of its tile is stored
                const GroupGemm &G = gs[k.gi];
                ok = ok && wait_count(p, p.ctl + CTL_TILES + G.tile_begin + k.tile,
                                      static_cast<unsigned int>(G.splits));
            }
            if (!epi_all(ok && t >= 0)) break;
            const GroupGemm &G = gs[k.gi];
            if (mma_task) {
                ++mj;
                st::tc_fence_after();
                const uint32_t acc = tmem + static_cast<uint32_t>(buf * GRP_BNMAX);
                if (G.splits == 1) {
                    epilogue_tma(G.g, &p.maps[k.gi].tmC, stage, acc, q, lane, k.m0, k.n0, 0, true, G.bn, &acc_empty[buf]);
                } else {
                    GemmArgs gp{};  // raw partial: no epilogue; TMA coordinate z2 = split
                    gp.M = G.g.M;
                    gp.N = G.g.N;
                    gp.c_grp = G.splits;
                    epilogue_tma(gp, &p.maps[k.gi].tmP, stage, acc, q, lane, k.m0, k.n0, k.split, true, G.bn, &acc_empty[buf]);
                }
                if (lane == 0) fence_proxy_async_global();  // this warp's stores have completed
                epi_bar();
                if (tid == 0) {
                    if (G.splits == 1) {
                        red_release_add(p.ctl + CTL_DONE + k.gi, 1u);
                    } else {
                        __threadfence();
                        red_release_add(p.ctl + CTL_TILES + G.tile_begin + k.tile, 1u);
                    }
                }
            } else {
                const int rows = BM / G.red_parts;
                group_reduce(G, k.m0 + k.part * rows, k.m0 + (k.part + 1) * rows, k.n0, tid);
                __threadfence();
                epi_bar();
                if (tid == 0) {
                    fence_proxy_async_global();
                    red_release_add(p.ctl + CTL_DONE + k.gi, 1u);
                }
            }
        }
    }
    st::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        st::tc_fence_after();
        st::tmem_dealloc(tmem, 2 * GRP_BNMAX);
    }
    if (threadIdx.x == 0) {  // the last CTA out leaves every counter at zero for the next launch
        __threadfence();
        if (atomicAdd(p.ctl + CTL_EXIT, 1u) == gridDim.x - 1) {
            for (int i = 0; i < p.ctl_words; i++) reinterpret_cast<volatile unsigned int *>(p.ctl)[i] = 0u;
            __threadfence();
        }
    }
}
