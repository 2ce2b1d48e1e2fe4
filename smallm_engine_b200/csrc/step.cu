// Persistent decode step: the whole token step (src/model/llama_model.cpp:148-177,
// src/model/qwen2_model.cpp:163-198) as ONE cooperative kernel.
//
// Why.  Batch-1 decode streams every weight byte once per token; what keeps
// it from the HBM roofline is the time HBM sits idle between dependent
// matrices (kernel boundaries, x staging, tails).  Here every SM keeps one
// resident CTA for the whole step, and the weight pieces of ALL the step's
// matrices stream, in order, through one shared-memory byte ring that never
// waits on a data dependency -- only on ring space: whichever warp frees a
// piece's space starts the copies of the next pieces that fit (ring_plan),
// so there is no producer warp and the 16 warps keep 128 registers each.  The
// warps walk the op list; between dependent ops they meet at a grid-wide
// barrier (a release counter in global memory), stage the new x and continue
// on pieces that are often already in shared memory.
//
// Ops, in order: EMBED, then per layer QKV -> ATTN -> O -> GATE/UP -> DOWN,
// then LM_HEAD + greedy argmax; the last CTA to finish advances the decode
// state (token, position, id list).  Each op ends with a grid barrier arrival
// ("signal"); an op that reads the previous ops' results first waits for the
// barrier count (counter >= signals so far x grid).  The counter is reset by
// the last CTA of the step, so a captured graph replays the kernel as is.
//
// GEMV ops (same block formats and fused epilogues as gemv.cuh): x is staged
// as three-digit block fixed point (gemv.cuh, XRec) and every consumer thread
// keeps the record of ONE 32-element unit of x in registers for the whole
// op ("x-stationary"): thread (warp w, lane l) owns unit u = (w % WS) * 32 + l
// of the row slot w / WS (WS = warps per row, ceil(units / 32)), and the RS
// = 16 / WS row slots of the CTA take RPT rows each of every piece.  A piece
// is R = RS * RPT consecutive rows (one contiguous range: one bulk copy).
// Per piece each warp reduces its RPT rows with shuffles, the partials meet
// in shared memory, and one warp (rotating with the piece) sums them and runs
// the fused epilogue.
//
// ATTN op (qwen2_model.cpp:111-133): split-K over (KV head, position range)
// items, one item per CTA; 16 warps x 128/hd sub-warps walk the item's
// positions with an online softmax; a CTA merges its warps in shared memory
// and, when a head has several items, the last of them (atomic ticket) merges
// the items' partials.  K/V rows are read straight from the cache (L2-coherent
// loads): the QKV op's epilogue wrote this step's row moments earlier.
//
// Every wait is bounded (~1 s of SM clock).  A wait that gives up raises bit
// 4 of the device error word and the model's abort flag; every other wait in
// the grid then returns at once, thread 0 waits (bounded) for the CTA's copies
// in flight, and the kernel ends.  The host reads the error word after the
// step and raises.
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "dequant.cuh"
#include "engine.h"
#include "gemv.cuh"
#include "model.h"

namespace smallm {

enum { SOP_EMBED = 0, SOP_GEMV = 1, SOP_ATTN = 2 };

constexpr int kStepW = 16;                    // consumer warps (one producer warp more)
constexpr int kStepThreads = (kStepW + 1) * 32;
constexpr uint32_t kStepSlots = 32;           // ring pieces in flight at most
constexpr uint32_t kStepPartRows = 64;        // rows of one piece's partials (R <= 64)
constexpr unsigned int kStepErrBit = 16u;
constexpr int kStepMaxGroup = 8;           // query heads per KV head

// One op of the step (device memory).  The GEMV output fields carry the same
// names as GemvParams so the fused epilogue (gemv_epilogue_row) reads them.
struct StepOp {
    uint32_t kind, fmt, pro, epi, wait, signal;
    uint32_t trace_kind, pad0;  // kind code of this op's slot in a traced step
    // GEMV: matrix and piece geometry
    const uint8_t* w;
    uint32_t row_stride, rows, rows_pad, cols, units;
    uint32_t ws, rs, rpt, prows, npieces;
    // GEMV inputs / fused epilogue outputs
    const float* x;
    const float* norm_w;
    float eps;
    float* y;
    const float* bias;
    uint32_t q_rows, k_rows, head_dim, max_ctx;
    float* qout;
    float* kcache;
    float* vcache;
    const float2* rope;
    const uint32_t* pos;
    unsigned long long* argmax;
    uint32_t row_offset;
    float* peer_out[kMaxTP];  // unused here (EPI_PEER is not a step op)
    uint32_t tp;
    // ATTN
    const float* q;
    float* out;
    float* part;               // [n_kv * S][G][hd + 2] item partials
    unsigned int* tickets;     // [n_kv], zero between steps
    uint32_t n_heads, n_kv;
    // EMBED
    QMat emb;
};

static_assert(sizeof(StepOp) % 8 == 0, "StepOp is copied in 8-byte words");

struct StepArgs {
    const StepOp* ops;
    uint32_t nops, nsig;       // ops, signalling ops
    DecodeState* st;
    uint32_t* ids;
    uint32_t ids_cap;
    unsigned int* bar;         // grid barrier counter (zero between steps)
    unsigned int* abort_flag;  // set when any wait of the step gave up
    unsigned int* err;         // device error word
    uint32_t xbytes, ring_bytes;
    TraceSlot* trace;          // [nops] in a traced step, else null
    unsigned long long* pieces;  // traced step: CTA 0's pieces [piece_cap][4], else null
    uint32_t piece_cap;
};

// ------------------------------------------------------------- waiting --

__device__ __forceinline__ void step_raise(const StepArgs& a) {
    atomicOr(a.err, kStepErrBit);
    *(volatile unsigned int*)a.abort_flag = 1u;
    __threadfence();
}

// The abort flag lives in global memory: a wait looks at it only once it has
// waited for ~2^16 cycles (~33 us), and then every 2^12 cycles, so a wait that
// completes normally never pays for that load.
constexpr long long kAbortLookAfter = 1ll << 16;
constexpr long long kGiveUp = 1ll << 31;  // ~1 s

__device__ __forceinline__ bool abort_seen(const unsigned int* abort_flag, long long waited, long long& next) {
    if (!abort_flag || waited < next) return false;
    next = waited + 4096;
    return *(const volatile unsigned int*)abort_flag != 0u;
}

// mbarrier phase wait, bounded (~2^31 cycles) and abandoned when the step's
// abort flag is up.
__device__ __forceinline__ bool step_wait(uint64_t* bar, uint32_t parity, const unsigned int* abort_flag) {
    const uint32_t addr = smem_u32(bar);
    const long long t0 = clock64();
    long long next = kAbortLookAfter;
    for (;;) {
        uint32_t ok;
        // no suspend-time hint: a suspended warp resumes late after the phase
        // completes, and these waits are on the piece pipeline's critical path
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
            : "=r"(ok)
            : "r"(addr), "r"(parity)
            : "memory");
        if (ok) return true;
        const long long waited = clock64() - t0;
        if (waited > kGiveUp || abort_seen(abort_flag, waited, next)) return false;
    }
}

// Grid barrier: wait until the counter reaches `target` (wrap-safe compare).
__device__ __forceinline__ bool grid_wait(const unsigned int* bar, unsigned int target,
                                          const unsigned int* abort_flag) {
    const long long t0 = clock64();
    long long next = kAbortLookAfter;
    for (;;) {
        unsigned int v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(bar) : "memory");
        if ((int)(v - target) >= 0) return true;
        const long long waited = clock64() - t0;
        if (waited > kGiveUp || abort_seen(abort_flag, waited, next)) return false;
    }
}

__device__ __forceinline__ void step_sync() {  // the consumer warps (the producer never joins)
    asm volatile("bar.sync 1, %0;" ::"n"(kStepW * 32) : "memory");
}

// ---------------------------------------------------------------- GEMV --

// The CTA's piece ring.  Pieces are issued in the step's order (op by op,
// this CTA's pieces p = blockIdx.x, + gridDim.x, ...) and retired in the same
// order; piece j uses slot j % kStepSlots.  Only the lane that holds the
// retire turn (retired == j) touches the issue state, so no lock is needed.
struct StepRing {
    uint32_t retired;  // pieces whose space is free again
    uint32_t issued;   // pieces whose copy has been started
    uint32_t freed[kStepSlots];  // j + 1 once piece j (slot j % kStepSlots) is done with
    uint32_t head;     // ring offset just past the newest issued piece
    uint32_t op, p;    // next piece to issue: op index and piece index
    // geometry of op `op` (read from global memory once per op)
    uint32_t kind, np, R, stride, rows_pad;
    const uint8_t* w;
    uint32_t pstart[kStepSlots];  // ring offset of each in-flight piece
};

// The CTA's shared state, at file scope so every access compiles to a
// shared-memory instruction (a pointer passed through a struct or a
// non-inlined call would become a generic one, which waits on the long
// scoreboard).
extern __shared__ __align__(128) uint8_t s_dyn[];  // x region (records / attention scratch), then the ring
__shared__ __align__(8) uint64_t s_full[kStepSlots];  // piece landed in the ring (count 1 + bytes)
__shared__ uint32_t s_cnt[kStepSlots * kStepW];       // warps of a row slot done with the piece
__shared__ uint32_t s_slots[kStepSlots];              // row slots done with the piece
__shared__ float s_part[kStepSlots * kStepPartRows];  // row partials of each piece in flight
__shared__ StepRing s_ring;
__shared__ float s_red[32];
__shared__ unsigned long long s_best[kStepW];
// the current op's descriptor (raw storage: StepOp has default member initializers)
__shared__ __align__(16) unsigned long long s_op_raw[sizeof(StepOp) / 8];
#define s_op (*reinterpret_cast<StepOp*>(s_op_raw))
__shared__ StepArgs s_args;
__shared__ int s_cta_dead;  // some wait of this CTA gave up (read after a barrier: CTA-uniform)
__shared__ int s_last_item;

__device__ __forceinline__ uint8_t* step_ring() { return s_dyn + s_args.xbytes; }

// Issue the next pieces while a slot is free and the ring has room for them
// (one lane, holding the retire turn).  Placement: a piece goes right after
// the newest one, or at offset 0 when it would run past the end; it may not
// overlap the span [tail, head) of pieces in flight (tail = oldest's start).
__device__ __forceinline__ void ring_load_op(const StepArgs& a, StepRing& r) {
    if (r.op >= a.nops) return;
    const StepOp* op = a.ops + r.op;
    r.kind = op->kind;
    r.np = op->npieces;
    r.R = op->prows;
    r.stride = op->row_stride;
    r.rows_pad = op->rows_pad;
    r.w = op->w;
}

// Plan the next pieces while a slot is free and the ring has room for them
// (the producer's lane 0): their ring offsets, sizes and sources go to
// s_plan_*, and the ring state advances as if they were issued.  Returns how
// many (at most 32: one per producer lane, which issue them at once).
__shared__ uint32_t s_plan_off[32], s_plan_bytes[32];
__shared__ const uint8_t* s_plan_src[32];

__device__ __forceinline__ uint32_t ring_plan() {
    const StepArgs& a = s_args;
    StepRing& r = s_ring;
    const uint32_t RB = a.ring_bytes;
    uint32_t n = 0;
    while (n < 32 && r.issued - r.retired < kStepSlots) {
        while (r.op < a.nops && (r.kind != SOP_GEMV || r.p >= r.np)) {
            ++r.op;
            r.p = blockIdx.x;
            ring_load_op(a, r);
        }
        if (r.op >= a.nops) break;
        const uint32_t R = r.R, stride = r.stride;
        const uint32_t bytes = min(R, r.rows_pad - r.p * R) * stride;
        const uint32_t off = r.head + bytes <= RB ? r.head : 0u;
        if (r.issued != r.retired) {
            const uint32_t tail = r.pstart[r.retired % kStepSlots];
            const bool clash = tail < r.head ? (off < r.head && tail < off + bytes)  // occupied [tail, head)
                                             : (off < r.head || off + bytes > tail); // [tail, RB) + [0, head)
            if (clash) break;
        }
        r.pstart[r.issued % kStepSlots] = off;
        r.head = off + bytes;
        s_plan_off[n] = off;
        s_plan_bytes[n] = bytes;
        s_plan_src[n] = r.w + (size_t)r.p * R * stride;
        ++n;
        ++r.issued;
        r.p += gridDim.x;
    }
    return n;
}

// Piece j is done (its slot's warps have read it, its epilogue has run): mark
// it for the producer, which retires pieces in order and reuses their space.
__device__ __forceinline__ void ring_mark_done(uint32_t j) {
    __threadfence_block();
    reinterpret_cast<volatile uint32_t*>(s_ring.freed)[j % kStepSlots] = j + 1;
}

// The producer warp's lane 0: retire the pieces marked done, in order, and
// start the copies of the next pieces that fit, until every piece of the step
// is issued and consumed.  A copy's issue can stall the issuing thread, which
// is why no consumer does it.  Gives up (bounded) when no piece retires for
// ~1 s or the step's abort flag is up, then waits for its copies in flight.
__device__ __forceinline__ void step_producer(int lane) {
    StepRing& r = s_ring;
    volatile uint32_t* fr = r.freed;
    const StepArgs& a = s_args;
    uint8_t* const ring = step_ring();
    long long t0 = clock64();
    long long next = kAbortLookAfter;
    bool dead = false;
    for (;;) {
        uint32_t n = 0, first = 0, state = 0;  // state: 1 all done, 2 gave up
        if (lane == 0) {
            uint32_t q = r.retired;
            while (q != r.issued && fr[q % kStepSlots] == q + 1) ++q;
            const bool progress = q != r.retired;
            r.retired = q;
            first = r.issued;
            n = ring_plan();
            if (r.op >= a.nops && r.retired == r.issued) {
                state = 1;  // all issued, all consumed
            } else if (progress || n) {
                t0 = clock64();
                next = kAbortLookAfter;
            } else {
                const long long waited = clock64() - t0;
                if (waited > kGiveUp || abort_seen(a.abort_flag, waited, next)) state = 2;
            }
        }
        __syncwarp();
        n = __shfl_sync(0xffffffffu, n, 0);
        first = __shfl_sync(0xffffffffu, first, 0);
        state = __shfl_sync(0xffffffffu, state, 0);
        if ((uint32_t)lane < n) {  // the planned copies, one per lane
            const uint32_t j = first + lane, s = j % kStepSlots;
            if (a.pieces && blockIdx.x == 0 && j < a.piece_cap) a.pieces[4 * j] = global_ns();
            mbar_arrive_expect_tx(&s_full[s], s_plan_bytes[lane]);
            bulk_g2s(ring + s_plan_off[lane], s_plan_src[lane], s_plan_bytes[lane], &s_full[s]);
        }
        __syncwarp();
        if (state == 1) break;
        if (state == 2) {
            dead = true;
            break;
        }
    }
    if (dead && lane == 0) {
        step_raise(a);
        for (uint32_t q2 = r.retired; q2 < r.issued; ++q2)
            step_wait(&s_full[q2 % kStepSlots], (q2 / kStepSlots) & 1u, nullptr);
    }
}

// x -> three-digit records of every 32-element block (times the norm weight
// when the RMSNorm is fused; its 1/rms is returned and applied per row).
template <class Fmt>
__device__ __forceinline__ float step_stage_x(const StepOp& op, int warp, int lane) {
    const int ctid = warp * 32 + lane;
    constexpr uint32_t kStride = kStepW * 32;
    constexpr int kB = 4;
    const uint32_t ngr = op.cols / 4;  // a multiple of 8: whole blocks
    const float4* x4 = reinterpret_cast<const float4*>(op.x);
    const float4* w4 = reinterpret_cast<const float4*>(op.norm_w);
    const bool rms = op.pro == PRO_RMS;
    float ss = 0.f;
    for (uint32_t g0 = 0; g0 < ngr; g0 += kB * kStride) {
        float4 xq[kB], wq[kB];
#pragma unroll
        for (int k = 0; k < kB; ++k) {
            const uint32_t g = g0 + ctid + k * kStride;
            const bool in = g < ngr;
            xq[k] = in ? __ldcg(x4 + g) : make_float4(0.f, 0.f, 0.f, 0.f);
            wq[k] = (in && rms) ? __ldg(w4 + g) : make_float4(1.f, 1.f, 1.f, 1.f);
        }
#pragma unroll
        for (int k = 0; k < kB; ++k) {
            // a warp whose first granule lies past the end has no block here
            // (warp-uniform, so the shuffles inside stay whole-warp)
            if (g0 + (uint32_t)warp * 32 + k * kStride >= ngr) continue;
            const uint32_t g = g0 + ctid + k * kStride;
            float4 q = xq[k];
            ss += q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w;
            q.x *= wq[k].x;
            q.y *= wq[k].y;
            q.z *= wq[k].z;
            q.w *= wq[k].w;
            build_xrec_lane<Fmt::XK>(q, lane, g < ngr, s_dyn + (size_t)(g >> 3) * kXrecBytes);
        }
    }
    if (rms) {
        ss = warp_sum(ss);
        if (lane == 0) s_red[warp] = ss;
    }
    step_sync();
    float inv = 1.0f;
    if (rms) {
        float t = 0.f;
#pragma unroll
        for (int k = 0; k < kStepW; ++k) t += s_red[k];
        inv = 1.0f / sqrtf(t / (float)op.cols + op.eps);  // ops::rmsnorm (ops.cpp:29-40)
    }
    return inv;
}

// Epilogue operands that do not depend on the row's dot product (rotary
// cos/sin, biases), loaded before the piece's partial sums are complete so
// their latency hides behind the other warps' work.
struct EpiPre {
    float2 cs;
    float b0, b1;
};

__device__ __forceinline__ EpiPre step_epi_pre(const StepOp& op, uint32_t row, uint32_t pos) {
    EpiPre e{make_float2(0.f, 0.f), 0.f, 0.f};
    if (op.epi != EPI_QKV || row >= op.rows) return e;
    const uint32_t hd = op.head_dim, half = hd >> 1;
    if (row < op.q_rows + op.k_rows) {
        if ((row & 1) == 0 && row + 1 < op.rows) {
            const bool isq = row < op.q_rows;
            const uint32_t pr = (isq ? row : row - op.q_rows) >> 1;  // rotary pair index
            const uint32_t ii = pr % half;
            e.cs = __ldg(op.rope + (size_t)pos * half + ii);
            if (op.bias) {
                const uint32_t la = (pr / half) * hd + ii, bo = isq ? 0u : op.q_rows;
                e.b0 = __ldg(op.bias + bo + la);
                e.b1 = __ldg(op.bias + bo + la + half);
            }
        }
    } else if (op.bias) {
        e.b0 = __ldg(op.bias + row);  // V rows follow Q and K in the bias vector too
    }
    return e;
}

// The fused epilogue of one finished row (v = W.x after 1/rms): the same
// arithmetic as gemv.cuh's, with the residual added by a single atomic add
// (each row is added once per op, so the sum is the plain f32 add) and the
// rotary/bias operands taken from `e`.
__device__ __forceinline__ void step_epilogue(const StepOp& op, uint32_t row, float v, float v_next,
                                              const EpiPre& e, unsigned long long& best) {
    switch (op.epi) {
        case EPI_STORE:
            if (row < op.rows) op.y[row] = v;
            break;
        case EPI_RESIDUAL:  // x += W.h (ops::axpy, qwen2_model.cpp:178,184)
            if (row < op.rows) atomicAdd(op.y + row, v);
            break;
        case EPI_SWIGLU: gemv_epilogue_row<EPI_SWIGLU>(op, row, v, v_next, best); break;
        case EPI_LOGITS: gemv_epilogue_row<EPI_LOGITS>(op, row, v, v_next, best); break;
        case EPI_QKV: {
            const uint32_t hd = op.head_dim, half = hd >> 1;
            const uint32_t pos = *op.pos;
            if (row < op.q_rows + op.k_rows) {
                if ((row & 1) == 0 && row + 1 < op.rows) {
                    const bool isq = row < op.q_rows;
                    const uint32_t pr = (isq ? row : row - op.q_rows) >> 1;
                    const uint32_t head = pr / half, ii = pr % half;
                    const uint32_t la = head * hd + ii, lb = la + half;
                    float x0 = v, x1 = v_next;
                    if (op.bias) {
                        x0 += e.b0;
                        x1 += e.b1;
                    }
                    // ops::rope (ops.cpp:84-89) with the reference build's fused rounding
                    const float o0 = fmaf(x0, e.cs.x, -__fmul_rn(x1, e.cs.y));
                    const float o1 = fmaf(x0, e.cs.y, __fmul_rn(x1, e.cs.x));
                    if (isq) {
                        op.qout[la] = o0;
                        op.qout[lb] = o1;
                    } else {
                        float* kr = op.kcache + ((size_t)head * op.max_ctx + pos) * hd;
                        kr[ii] = o0;
                        kr[ii + half] = o1;
                    }
                }
            } else if (row < op.rows) {
                const uint32_t lv = row - op.q_rows - op.k_rows;
                float vv = v;
                if (op.bias) vv += e.b0;
                op.vcache[((size_t)(lv / hd) * op.max_ctx + pos) * hd + lv % hd] = vv;
            }
            break;
        }
        default: break;
    }
}

// This CTA's position in its piece sequence (piece counter j and ring
// placement head, identical to ring_plan's), the abandon flag and the
// greedy-argmax key of a logits op.
struct PieceCursor {
    uint32_t j, head, dead;
    unsigned long long best;
};

// One GEMV op (rows per slot op.rpt <= 4: the row loop and the shuffle
// reduction run for 4 rows, the missing ones as zeros).
template <class Fmt>
__device__ __forceinline__ PieceCursor step_gemv(int warp, int lane, PieceCursor cur) {
    constexpr int RPT = Fmt::STEP_RPT;  // rows per slot at most (register budget)
    constexpr int LPR = 32 / RPT;
    const StepOp& op = s_op;
    const StepArgs& a = s_args;
    uint8_t* const ring = step_ring();
    const unsigned int* const abort_flag = a.abort_flag;
    const uint32_t RB = a.ring_bytes;
    uint32_t j = cur.j, head = cur.head;
    bool dead = cur.dead != 0;
    unsigned long long best = cur.best;
    const float inv = step_stage_x<Fmt>(op, warp, lane);
    // A piece is R = RS * rpt consecutive rows (one bulk copy of ~32 KB: the
    // per-SM copy engine needs copies that large to keep up with HBM); row
    // slot `slot` (WS warps, one unit of x per lane) takes its rpt rows.
    const uint32_t U = op.units, WS = op.ws, RS = op.rs, R = op.prows, stride = op.row_stride, rpt = op.rpt;
    const uint32_t slot = (uint32_t)warp / WS, wi = (uint32_t)warp % WS;
    const bool active = slot < RS;
    const uint32_t u = wi * 32 + (uint32_t)lane;
    const uint32_t r0 = slot * rpt;  // this slot's first row in a piece
    const uint32_t pos_op = op.epi == EPI_QKV ? *op.pos : 0u;  // the step's position (RoPE row)
    const uint32_t npieces = op.npieces, rows_pad = op.rows_pad;
    for (uint32_t p = blockIdx.x; p < npieces; p += gridDim.x, ++j) {
        const uint32_t rows_here = min(R, rows_pad - p * R);
        const uint32_t bytes = rows_here * stride;
        const uint32_t off = head + bytes <= RB ? head : 0u;  // the ring placement, as ring_plan makes it
        head = off + bytes;
        if (!active) continue;
        const uint32_t s = j % kStepSlots, ph = (j / kStepSlots) & 1u;
        if (!dead && !step_wait(&s_full[s], ph, abort_flag)) {
            dead = true;
            step_raise(a);
        }
        dead = __any_sync(0xffffffffu, dead);  // warp-uniform (the shuffles below)
        const bool stamp = a.pieces && blockIdx.x == 0 && lane == 0 && j < a.piece_cap;
        if (stamp && warp == 0) a.pieces[4 * j + 1] = global_ns();
        float acc[RPT];
#pragma unroll
        for (int k = 0; k < RPT; ++k) acc[k] = 0.f;
        if (u < U && r0 < rows_here && !dead) {
            XRec xr;  // this thread's unit of x (three-digit record)
            load_xrec(s_dyn, u, xr);
            const uint8_t* base = ring + off + (size_t)r0 * stride;
#pragma unroll
            for (int k = 0; k < RPT; ++k) {
                if ((uint32_t)k < rpt && r0 + k < rows_here) {
                    typename Fmt::Raw raw;
                    Fmt::load(base + (size_t)k * stride, u, U, raw);
                    acc[k] = Fmt::dot(raw, 0, xr, u);
                }
            }
        }
        // lanes k*LPR .. k*LPR + LPR-1 end with this warp's part of row k
        const float v = warp_reduce_rows<RPT>(acc, lane);
        if ((lane % LPR) == 0 && (uint32_t)lane / LPR < rpt)
            s_part[s * kStepPartRows + (r0 + lane / LPR) * WS + wi] = v;
        __syncwarp();
        // the slot's last warp to finish closes the slot's rows, and the last
        // slot to close hands the piece back: no warp waits for another
        uint32_t last = 1u;
        if (WS > 1) {
            if (lane == 0) {
                __threadfence_block();
                last = atomicAdd(&s_cnt[s * kStepW + slot], 1u) == WS - 1 ? 1u : 0u;
            }
            last = __shfl_sync(0xffffffffu, last, 0);
        }
        if (!last) continue;
        __threadfence_block();
        if (lane == 0) s_cnt[s * kStepW + slot] = 0u;
        {
            const uint32_t r = r0 + (uint32_t)lane;  // lanes 0..rpt-1: this slot's rows
            float val = 0.f;
            if ((uint32_t)lane < rpt)
                for (uint32_t k = 0; k < WS; ++k) val += s_part[s * kStepPartRows + r * WS + k];
            val *= inv;  // 1/rms of the fused RMSNorm (1 if plain)
            const float v_next = __shfl_down_sync(0xffffffffu, val, 1);  // partner row of a pair
            if ((uint32_t)lane < rpt && r < rows_here && !dead) {
                const EpiPre e = step_epi_pre(op, p * R + r, pos_op);
                step_epilogue(op, p * R + r, val, v_next, e, best);
            }
        }
        __syncwarp();
        if (lane == 0) {
            __threadfence_block();
            const bool piece_done = RS == 1 || atomicAdd(&s_slots[s], 1u) == RS - 1;
            if (piece_done) {
                if (RS > 1) s_slots[s] = 0u;
                if (stamp) a.pieces[4 * j + 2] = global_ns();
                if (!dead) ring_mark_done(j);
                if (stamp) a.pieces[4 * j + 3] = global_ns();
            }
        }
    }
    return PieceCursor{j, head, dead ? 1u : 0u, best};
}


// ----------------------------------------------------------- attention --

// Online-softmax state of one head over some positions: running max m, sum
// of exp(score - m) l, unnormalised output o (4 dims of one lane).
__device__ __forceinline__ void attn_merge(float& m, float& l, float4& o, float m2, float l2, float4 o2) {
    const float M = fmaxf(m, m2);
    const float a1 = M == -INFINITY ? 0.f : expf(m - M);
    const float a2 = M == -INFINITY ? 0.f : expf(m2 - M);
    l = a1 * l + a2 * l2;
    o.x = a1 * o.x + a2 * o2.x;
    o.y = a1 * o.y + a2 * o2.y;
    o.z = a1 * o.z + a2 * o2.z;
    o.w = a1 * o.w + a2 * o2.w;
    m = M;
}

// One attention item per CTA: KV head kvh, positions [b, e).  The op's
// barrier (on the QKV op) is taken in here: the item's first batch of cached
// K/V rows (every position but the newest, which this step's QKV op writes)
// is loaded before it, so that latency overlaps the wait.
template <int HD>
__device__ __forceinline__ uint32_t step_attn(int warp, int lane, uint32_t dead_in, uint32_t target) {
    const StepOp& op = s_op;
    const StepArgs& a = s_args;
    constexpr int RPI = 128 / HD;            // positions per warp instruction (sub-warps)
    constexpr int LPR = 32 / RPI;            // lanes per position: 4 dims each
    constexpr int kHP = 4;                   // heads per pass (register budget)
    constexpr int kB = 2;                    // positions per position-lane and load batch (registers)
    constexpr uint32_t SR = HD + 4;          // scratch row: HD outputs, max, sum, pad to 16 bytes
    constexpr uint32_t NRL = kStepW * RPI;   // position lanes of the CTA
    const int ctid = warp * 32 + lane;
    const uint32_t G = op.n_heads / op.n_kv;
    const uint32_t n = min(*op.pos + 1, op.max_ctx);  // fixed for the whole step
    const uint32_t newest = n - 1;
    // items of at most one load batch of positions each, as many as the grid allows
    uint32_t smax = gridDim.x / op.n_kv;
    if (smax < 1) smax = 1;
    uint32_t S = (n + NRL * kB - 1) / (NRL * kB);
    if (S > smax) S = smax;
    if (S < 1) S = 1;
    const uint32_t L = (n + S - 1) / S;
    const uint32_t item = blockIdx.x;
    const bool has = item < op.n_kv * S;
    const uint32_t kvh = has ? item / S : 0u, sidx = has ? item % S : 0u;
    const uint32_t b = sidx * L, e = has ? min(n, b + L) : 0u;
    const int sub = lane / LPR, dl = lane % LPR;
    const float* kb = op.kcache + (size_t)kvh * op.max_ctx * HD;
    const float* vb = op.vcache + (size_t)kvh * op.max_ctx * HD;
    const uint32_t first = b + (uint32_t)warp * RPI;
    uint32_t trips = first < e ? (e - first + NRL - 1) / NRL : 0u;  // warp-uniform
    float4 kk[kB], vv[kB];
    auto load_batch = [&](uint32_t i, bool cached_only) {
#pragma unroll
        for (int c = 0; c < kB; ++c) {
            const uint32_t t = first + (i + c) * NRL + (uint32_t)sub;
            const bool in = i + c < trips && t < e && !(cached_only && t == newest);
            if (in) {
                kk[c] = __ldcg(reinterpret_cast<const float4*>(kb + (size_t)t * HD) + dl);
                vv[c] = __ldcg(reinterpret_cast<const float4*>(vb + (size_t)t * HD) + dl);
            } else if (!cached_only || i + c >= trips || t >= e) {
                kk[c] = make_float4(0.f, 0.f, 0.f, 0.f);
                vv[c] = kk[c];
            }
        }
    };
    load_batch(0, true);
    // the QKV op's results (q, the newest K/V row) are complete past this barrier
    bool dead = dead_in != 0;
    if (ctid == 0 && !dead && !grid_wait(a.bar, target, a.abort_flag)) {
        s_cta_dead = 1;
        step_raise(a);
    }
    step_sync();
    dead = s_cta_dead != 0;
    if (dead) trips = 0u;
#pragma unroll
    for (int c = 0; c < kB; ++c) {
        const uint32_t t = first + c * NRL + (uint32_t)sub;
        if ((uint32_t)c < trips && t == newest) {
            kk[c] = __ldcg(reinterpret_cast<const float4*>(kb + (size_t)t * HD) + dl);
            vv[c] = __ldcg(reinterpret_cast<const float4*>(vb + (size_t)t * HD) + dl);
        }
    }
    const float scale = 1.0f / sqrtf((float)HD);
    float* scr = reinterpret_cast<float*>(s_dyn);  // [kStepW][G][SR]
    for (uint32_t h0 = 0; h0 < G; h0 += kHP) {
        float4 qv[kHP];
        float m[kHP], l[kHP];
        float4 o[kHP];
#pragma unroll
        for (int h = 0; h < kHP; ++h) {
            qv[h] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (has && h0 + h < G)
                qv[h] = __ldcg(reinterpret_cast<const float4*>(op.q + ((size_t)kvh * G + h0 + h) * HD) + dl);
            m[h] = -INFINITY;
            l[h] = 0.f;
            o[h] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        for (uint32_t i = 0; i < trips; i += kB) {
            if (i > 0 || (h0 > 0 && trips > (uint32_t)kB)) load_batch(i, false);  // batch 0 is still in registers otherwise
            bool ok[kB];
#pragma unroll
            for (int c = 0; c < kB; ++c) ok[c] = i + c < trips && first + (i + c) * NRL + (uint32_t)sub < e;
#pragma unroll
            for (int c = 0; c < kB; ++c) {
                if (i + c >= trips) break;  // warp-uniform
#pragma unroll
                for (int h = 0; h < kHP; ++h) {
                    if (h0 + h >= G) break;  // uniform
                    float sc = qv[h].x * kk[c].x + qv[h].y * kk[c].y + qv[h].z * kk[c].z + qv[h].w * kk[c].w;
#pragma unroll
                    for (int off = 1; off < LPR; off <<= 1) sc += __shfl_xor_sync(0xffffffffu, sc, off);
                    sc *= scale;
                    if (ok[c]) {
                        const float mn = fmaxf(m[h], sc);
                        const float co = expf(m[h] - mn);  // 0 for the first position (m = -inf)
                        const float pr = expf(sc - mn);
                        l[h] = l[h] * co + pr;
                        o[h].x = o[h].x * co + pr * vv[c].x;
                        o[h].y = o[h].y * co + pr * vv[c].y;
                        o[h].z = o[h].z * co + pr * vv[c].z;
                        o[h].w = o[h].w * co + pr * vv[c].w;
                        m[h] = mn;
                    }
                }
            }
        }
        // merge the sub-warps (same dims, other positions)
#pragma unroll
        for (int off = LPR; off < 32; off <<= 1) {
#pragma unroll
            for (int h = 0; h < kHP; ++h) {
                const float m2 = __shfl_xor_sync(0xffffffffu, m[h], off);
                const float l2 = __shfl_xor_sync(0xffffffffu, l[h], off);
                float4 o2;
                o2.x = __shfl_xor_sync(0xffffffffu, o[h].x, off);
                o2.y = __shfl_xor_sync(0xffffffffu, o[h].y, off);
                o2.z = __shfl_xor_sync(0xffffffffu, o[h].z, off);
                o2.w = __shfl_xor_sync(0xffffffffu, o[h].w, off);
                attn_merge(m[h], l[h], o[h], m2, l2, o2);
            }
        }
        if (sub == 0) {
#pragma unroll
            for (int h = 0; h < kHP; ++h) {
                if (h0 + h >= G) break;
                float* r = scr + ((size_t)warp * G + h0 + h) * SR;  // SR floats: 16-byte rows
                reinterpret_cast<float4*>(r)[dl] = o[h];
                if (dl == 0) {
                    r[HD] = m[h];
                    r[HD + 1] = l[h];
                }
            }
        }
    }
    step_sync();
    // merge the 16 warps: thread -> (head, dim)
    float* part = op.part + (size_t)(kvh * S + sidx) * G * (HD + 2);
    if (has && !dead) {
        for (uint32_t idx = ctid; idx < G * HD; idx += kStepW * 32) {
            const uint32_t h = idx / HD, d = idx % HD;
            float M = -INFINITY;
            for (int w = 0; w < kStepW; ++w) M = fmaxf(M, scr[((size_t)w * G + h) * SR + HD]);
            float O = 0.f, Ls = 0.f;
            if (M != -INFINITY) {
                for (int w = 0; w < kStepW; ++w) {
                    const float* r = scr + ((size_t)w * G + h) * SR;
                    const float wt = expf(r[HD] - M);  // 0 for a warp without positions
                    O = fmaf(wt, r[d], O);
                    Ls = fmaf(wt, r[HD + 1], Ls);
                }
            }
            if (S == 1) {
                op.out[((size_t)kvh * G + h) * HD + d] = O / Ls;
            } else {
                part[(size_t)h * (HD + 2) + d] = O;
                if (d == 0) {
                    part[(size_t)h * (HD + 2) + HD] = M;
                    part[(size_t)h * (HD + 2) + HD + 1] = Ls;
                }
            }
        }
    }
    if (S > 1) {
        // the last item of this KV head merges all of its items
        __threadfence();
        step_sync();
        if (ctid == 0) s_last_item = (has && !dead) ? (atomicAdd(op.tickets + kvh, 1u) == S - 1 ? 1 : 0) : 0;
        step_sync();
        if (s_last_item) {
            __threadfence();
            const float* hp = op.part + (size_t)kvh * S * G * (HD + 2);
            for (uint32_t idx = ctid; idx < G * HD; idx += kStepW * 32) {
                const uint32_t h = idx / HD, d = idx % HD;
                float M = -INFINITY;
                for (uint32_t s2 = 0; s2 < S; ++s2) M = fmaxf(M, __ldcg(hp + ((size_t)s2 * G + h) * (HD + 2) + HD));
                float O = 0.f, Ls = 0.f;
                for (uint32_t s2 = 0; s2 < S; ++s2) {
                    const float* r = hp + ((size_t)s2 * G + h) * (HD + 2);
                    const float mm = __ldcg(r + HD);
                    const float wt = mm == -INFINITY ? 0.f : expf(mm - M);
                    O = fmaf(wt, __ldcg(r + d), O);
                    Ls = fmaf(wt, __ldcg(r + HD + 1), Ls);
                }
                op.out[((size_t)kvh * G + h) * HD + d] = O / Ls;
            }
            if (ctid == 0) op.tickets[kvh] = 0u;
        }
    }
    step_sync();  // the scratch (x region) is reused by the next op
    return dead ? 1u : 0u;
}

// -------------------------------------------------------------- kernel --

template <class FA, class FB, int HD>
__global__ void __launch_bounds__(kStepThreads, 1) smallm_step_kernel(const StepArgs args) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        s_args = args;
        for (uint32_t s = 0; s < kStepSlots; ++s) {
            mbar_init(&s_full[s], 1);
            s_slots[s] = 0u;
        }
        for (uint32_t q = 0; q < kStepSlots * kStepW; ++q) s_cnt[q] = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        StepRing& r = s_ring;
        r.retired = r.issued = r.head = 0u;
        for (uint32_t q = 0; q < kStepSlots; ++q) r.freed[q] = 0u;
        r.op = 0u;
        r.p = blockIdx.x;
        ring_load_op(s_args, r);
        s_cta_dead = 0;
    }
    __syncthreads();
    if (warp == kStepW) {  // the producer: weights depend on nothing, so it streams ahead
        step_producer(lane);
        return;
    }
    const StepArgs& a = s_args;

    const int ctid = tid;
    uint32_t j = 0, head = 0, nsig = 0;
    bool dead = false;
    for (uint32_t k = 0; k < a.nops; ++k) {
        // this op's descriptor into shared memory (8-byte words)
        if (dead) s_cta_dead = 1;
        step_sync();
        for (uint32_t i = ctid; i < sizeof(StepOp) / 8; i += kStepW * 32)
            s_op_raw[i] =
                __ldg(reinterpret_cast<const unsigned long long*>(a.ops + k) + i);
        step_sync();
        dead = s_cta_dead != 0;
        const StepOp& op = s_op;
        TraceSlot* slot = a.trace ? a.trace + k : nullptr;
        if (ctid == 0) trace_mark(slot, 0);
        if (op.wait && op.kind != SOP_ATTN) {  // CTA-uniform: every thread reaches the barrier below
            if (ctid == 0 && !dead && !grid_wait(a.bar, nsig * gridDim.x, a.abort_flag)) {
                s_cta_dead = 1;
                step_raise(a);
            }
            step_sync();
            dead = s_cta_dead != 0;
        }
        if (ctid == 0) trace_mark(slot, 1);
        if (op.kind == SOP_GEMV) {
            PieceCursor cur{j, head, dead ? 1u : 0u, 0ull};
            if (op.fmt == 0) cur = step_gemv<FA>(warp, lane, cur);
            else cur = step_gemv<FB>(warp, lane, cur);
            j = cur.j;
            head = cur.head;
            dead = cur.dead != 0;
            unsigned long long best = cur.best;
            if (op.epi == EPI_LOGITS) {
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
                    best = other > best ? other : best;
                }
                if (lane == 0) s_best[warp] = best;
                step_sync();
                if (ctid == 0) {
                    unsigned long long b = 0ull;
                    for (int w = 0; w < kStepW; ++w) b = s_best[w] > b ? s_best[w] : b;
                    if (b && !dead) atomicMax(op.argmax, b);
                }
            }
        } else if (op.kind == SOP_ATTN) {
            // takes the op's barrier itself, after loading cached K/V rows
            const uint32_t d = dead ? 1u : 0u, target = nsig * gridDim.x;
            dead = step_attn<HD>(warp, lane, d, target) != 0u;
        } else if (op.kind == SOP_EMBED && !dead) {
            uint32_t tok = a.st->token;
            if (tok >= op.emb.rows) tok = 0;  // the host validates ids; never read outside the table
            const uint32_t ng = op.emb.cols / 32;
            for (uint32_t g = blockIdx.x + ctid * gridDim.x; g < ng; g += kStepW * 32 * gridDim.x)
                dequant_group(op.emb, tok, g, op.y + (size_t)g * 32);
            if (blockIdx.x == 0 && ctid == 0) a.st->argmax = 0ull;
        }
        if (op.signal) {
            step_sync();  // every warp's writes of this op are issued
            if (ctid == 0) trace_mark(slot, 2);
            if (ctid == 0) {
                __threadfence();
                const unsigned int old = atomicAdd(a.bar, 1u);
                if (k + 1 == a.nops && old == a.nsig * gridDim.x - 1u && !dead) {
                    // the step's last CTA: advance the decode state
                    __threadfence();
                    const unsigned long long key = *(volatile unsigned long long*)&a.st->argmax;
                    const uint32_t tok = argmax_key_index(key);
                    DecodeState* st = a.st;
                    st->token = tok;
                    if (a.ids && st->step < a.ids_cap) a.ids[st->step] = tok;
                    st->step += 1;
                    st->pos += 1;
                    *a.bar = 0u;
                }
            }
            ++nsig;
        }
    }
    // (a CTA whose wait gave up leaves its copies in flight to the producer,
    // which waits for them before it returns: the CTA stays until then)
}

// ---------------------------------------------------------------- host --

template <int HD>
static const void* step_kernel_hd(uint32_t fa, uint32_t fb) {
    if (fa == SM_T_Q4_0 && fb == SM_T_Q8_0) return (const void*)smallm_step_kernel<FmtQ4_0, FmtQ8_0, HD>;
    if (fa == SM_T_Q8_0 && fb == SM_T_Q8_0) return (const void*)smallm_step_kernel<FmtQ8_0, FmtQ8_0, HD>;
    if (fa == SM_T_Q4_0 && fb == SM_T_Q4_0) return (const void*)smallm_step_kernel<FmtQ4_0, FmtQ4_0, HD>;
    if (fa == SM_T_Q8_0 && fb == SM_T_Q4_0) return (const void*)smallm_step_kernel<FmtQ8_0, FmtQ4_0, HD>;
    return nullptr;
}

static const void* step_kernel_for(uint32_t fa, uint32_t fb, uint32_t hd) {
    if (hd == 128) return step_kernel_hd<128>(fa, fb);
    if (hd == 64) return step_kernel_hd<64>(fa, fb);
    if (hd == 32) return step_kernel_hd<32>(fa, fb);
    return nullptr;
}

// Why the persistent step cannot run this model ("" if it can).
std::string Model::step_unsupported() const {
    if (tp_size != 1) return "tensor parallel";
    if (n_layers == 0) return "no layers";
    const uint32_t fa = layers[0].qkv.type;
    for (const LayerW& L : layers) {
        if (!L.fused_v) return "separate V matrix";
        for (const QMat* m : {&L.qkv, &L.o, &L.gu, &L.down})
            if (m->type != fa) return "mixed layer formats";
    }
    if (!step_kernel_for(fa, out_m.type, hd)) return "weight formats or head_dim";
    if (embd_m.type != SM_T_Q4_0 && embd_m.type != SM_T_Q8_0 && embd_m.type != SM_T_F32 && embd_m.type != SM_T_Q4_K &&
        embd_m.type != SM_T_Q6_K)
        return "embedding format";
    if (hd != 32 && hd != 64 && hd != 128) return "head_dim";
    if (nh_l % nkv_l || nh_l / nkv_l > (uint32_t)kStepMaxGroup) return "head grouping";
    for (const QMat* m : {&layers[0].qkv, &layers[0].o, &layers[0].gu, &layers[0].down, &out_m})
        if (m->units > 32u * kStepW) return "rows longer than the step's x registers";
    // opt-in while the per-op kernels are faster on the measured workloads
    const char* want = std::getenv("SMALLM_STEP");
    if (!want || std::strcmp(want, "persistent") != 0) return "per-op kernels (SMALLM_STEP=persistent selects it)";
    return "";
}

void Model::build_step() {
    step_on = false;
    step_why = step_unsupported();
    if (!step_why.empty()) return;
    const void* fn = step_kernel_for(layers[0].qkv.type, out_m.type, hd);
    cudaFuncAttributes fa{};
    SM_CUDA(cudaFuncGetAttributes(&fa, fn));
    int dev = 0, optin = 0;
    SM_CUDA(cudaGetDevice(&dev));
    SM_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    const size_t dyn_max = (size_t)optin - fa.sharedSizeBytes;

    // x region: the largest op's records, or the attention's per-warp scratch
    const uint32_t G = nh_l / nkv_l;
    size_t xbytes = (size_t)kStepW * G * (hd + 4) * 4;
    for (const QMat* m : {&layers[0].qkv, &layers[0].o, &layers[0].gu, &layers[0].down, &out_m})
        xbytes = std::max(xbytes, (size_t)m->units * kXrecBytes);
    xbytes = (xbytes + 127) / 128 * 128;
    if (xbytes + 64 * 1024 > dyn_max) {
        step_why = "shared memory";
        return;
    }
    const size_t ring = (dyn_max - xbytes) / 128 * 128;

    // piece geometry of a matrix: WS warps per row, RS row slots, RPT rows
    // per slot (R = RS * RPT rows per piece, even, at most 64, a piece at most
    // `cap` bytes: 40 KB, or SMALLM_STEP_PIECE_KB, and a third of the ring)
    size_t cap = ring / 3;
    if (const char* e = std::getenv("SMALLM_STEP_PIECE_KB")) cap = std::min(cap, (size_t)std::atoi(e) * 1024);
    else cap = std::min(cap, (size_t)40 * 1024);
    auto geometry = [&](const QMat& m, StepOp& op) {
        // WS warps cover a row's units (one per lane); RS = 16 / WS row slots
        // take rpt rows each of every piece (rpt even: rotary and SwiGLU row
        // pairs stay in one slot), so a piece is R = RS * rpt rows in one
        // copy, at most `cap` bytes and a third of the ring
        const uint32_t WS = (m.units + 31) / 32;
        const uint32_t RS = kStepW / WS;
        uint32_t rpt = m.type == SM_T_Q4_0 ? FmtQ4_0::STEP_RPT : FmtQ8_0::STEP_RPT;
        while (rpt > 2 && (size_t)RS * rpt * m.row_stride > cap) rpt /= 2;
        if (RS == 0 || rpt < 2 || RS * rpt * WS > kStepPartRows ||
            (size_t)RS * rpt * m.row_stride > ring / 3)
            throw Error(1, "persistent step: no piece geometry for a matrix of " + std::to_string(m.cols) + " columns");
        op.w = m.base;
        op.row_stride = m.row_stride;
        op.rows = m.rows;
        op.rows_pad = m.rows_pad;
        op.cols = m.cols;
        op.units = m.units;
        op.ws = WS;
        op.rs = RS;
        op.rpt = rpt;
        op.prows = RS * rpt;
        op.npieces = (m.rows_pad + op.prows - 1) / op.prows;
    };

    std::vector<StepOp> ops;
    auto blank = [] {
        StepOp o;
        std::memset(&o, 0, sizeof(o));
        return o;
    };
    {
        StepOp e = blank();
        e.kind = SOP_EMBED;
        e.trace_kind = 1;
        e.signal = 1;
        e.emb = embd_m;
        e.y = x;
        ops.push_back(e);
    }
    const uint32_t qrows = nh_l * hd, krows = nkv_l * hd;
    for (uint32_t i = 0; i < n_layers; ++i) {
        LayerW& L = layers[i];
        float* kc = kv + (size_t)(2 * i) * nkv_l * max_ctx * hd;
        float* vc = kv + (size_t)(2 * i + 1) * nkv_l * max_ctx * hd;
        StepOp g = blank();
        g.kind = SOP_GEMV;
        g.wait = g.signal = 1;
        g.pro = PRO_RMS;
        g.epi = EPI_QKV;
        g.trace_kind = 2;
        geometry(L.qkv, g);
        g.x = x;
        g.norm_w = L.attn_norm;
        g.eps = eps;
        g.bias = L.bias;
        g.q_rows = qrows;
        g.k_rows = krows;
        g.head_dim = hd;
        g.max_ctx = max_ctx;
        g.qout = q;
        g.kcache = kc;
        g.vcache = vc;
        g.rope = rope;
        g.pos = &st->pos;
        ops.push_back(g);

        StepOp t = blank();
        t.kind = SOP_ATTN;
        t.trace_kind = 4;
        t.wait = t.signal = 1;
        t.q = q;
        t.kcache = kc;
        t.vcache = vc;
        t.out = att;
        t.part = step_part;
        t.tickets = step_tickets;
        t.n_heads = nh_l;
        t.n_kv = nkv_l;
        t.head_dim = hd;
        t.max_ctx = max_ctx;
        t.pos = &st->pos;
        ops.push_back(t);

        StepOp o = blank();
        o.kind = SOP_GEMV;
        o.wait = o.signal = 1;
        o.pro = PRO_PLAIN;
        o.epi = EPI_RESIDUAL;
        o.trace_kind = 5;
        geometry(L.o, o);
        o.x = att;
        o.y = x;
        ops.push_back(o);

        StepOp u = blank();
        u.kind = SOP_GEMV;
        u.wait = u.signal = 1;
        u.pro = PRO_RMS;
        u.epi = EPI_SWIGLU;
        u.trace_kind = 6;
        geometry(L.gu, u);
        u.x = x;
        u.norm_w = L.ffn_norm;
        u.eps = eps;
        u.y = hbuf;
        ops.push_back(u);

        StepOp d = blank();
        d.kind = SOP_GEMV;
        d.wait = d.signal = 1;
        d.pro = PRO_PLAIN;
        d.epi = EPI_RESIDUAL;
        d.trace_kind = 7;
        geometry(L.down, d);
        d.x = hbuf;
        d.y = x;
        ops.push_back(d);
    }
    {
        StepOp h = blank();
        h.kind = SOP_GEMV;
        h.fmt = 1;
        h.wait = h.signal = 1;
        h.pro = PRO_RMS;
        h.epi = EPI_LOGITS;
        h.trace_kind = 8;
        geometry(out_m, h);
        h.x = x;
        h.norm_w = out_norm;
        h.eps = eps;
        h.y = logits_local;
        h.argmax = &st->argmax;
        h.row_offset = v0;
        ops.push_back(h);
    }
    step_ops = static_cast<StepOp*>(dalloc(sizeof(StepOp) * ops.size()));
    SM_CUDA(cudaMemcpy(step_ops, ops.data(), sizeof(StepOp) * ops.size(), cudaMemcpyHostToDevice));
    step_nops = (uint32_t)ops.size();
    step_nsig = 0;
    for (const StepOp& o : ops) step_nsig += o.signal;
    step_xbytes = (uint32_t)xbytes;
    step_ring = (uint32_t)ring;
    step_smem = xbytes + ring;
    step_fn = fn;
    set_smem_limit_once(fn, (int)step_smem);
    int per_sm = 0;
    SM_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kStepThreads, step_smem));
    if (per_sm < 1) {
        step_why = "occupancy";
        return;
    }
    step_grid = (uint32_t)sm_count;
    step_on = true;
}

// Per-model device buffers of the persistent step (made at load).
void Model::alloc_step_buffers() {
    const uint32_t G = nkv_l ? nh_l / nkv_l : 1;
    step_part = static_cast<float*>(dalloc(4ull * (size_t)sm_count * G * (hd + 2)));
    step_tickets = static_cast<unsigned int*>(dalloc(4ull * std::max(1u, nkv_l)));
    step_bar = static_cast<unsigned int*>(dalloc(64));
    step_abort = step_bar + 1;
    SM_CUDA(cudaMemsetAsync(step_tickets, 0, 4ull * std::max(1u, nkv_l), stream));
    SM_CUDA(cudaMemsetAsync(step_bar, 0, 64, stream));
}

void Model::launch_step(cudaStream_t s, TraceSlot* trace, unsigned long long* pieces, uint32_t piece_cap) {
    StepArgs a;
    a.ops = step_ops;
    a.nops = step_nops;
    a.nsig = step_nsig;
    a.st = st;
    a.ids = ids;
    a.ids_cap = ids_cap;
    a.bar = step_bar;
    a.abort_flag = step_abort;
    a.err = device_error_flag();
    a.xbytes = step_xbytes;
    a.ring_bytes = step_ring;
    a.trace = trace;
    a.pieces = pieces;
    a.piece_cap = piece_cap;
    void* args[] = {&a};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(step_grid);
    cfg.blockDim = dim3(kStepThreads);
    cfg.dynamicSmemBytes = step_smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: they wait on one another
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    SM_CUDA(cudaLaunchKernelExC(&cfg, step_fn, args));
}

// One step of the persistent kernel with per-op timestamps (earliest CTA at
// the op's start, earliest past its barrier wait, latest at its end); the
// slots' kind codes follow the per-op kernels' trace kinds.
void Model::trace_step_persistent(uint32_t token, uint32_t pos, std::vector<TraceSlot>& out) {
    constexpr uint32_t kPieceCap = 8192;
    if (!trace_dev_step) {
        trace_dev_step = static_cast<TraceSlot*>(dalloc(sizeof(TraceSlot) * step_nops));
        trace_dev_pieces = static_cast<unsigned long long*>(dalloc(32ull * kPieceCap));
    }
    std::vector<StepOp> ops(step_nops);
    SM_CUDA(cudaMemcpy(ops.data(), step_ops, sizeof(StepOp) * step_nops, cudaMemcpyDeviceToHost));
    std::vector<TraceSlot> init(step_nops);
    for (uint32_t k = 0; k < step_nops; ++k) init[k] = TraceSlot{~0ull, ~0ull, 0ull, ops[k].trace_kind};
    SM_CUDA(cudaMemcpyAsync(trace_dev_step, init.data(), sizeof(TraceSlot) * step_nops, cudaMemcpyHostToDevice,
                            stream));
    SM_CUDA(cudaMemsetAsync(trace_dev_pieces, 0, 32ull * kPieceCap, stream));
    set_state(token, pos);
    launch_step(stream, trace_dev_step, trace_dev_pieces, kPieceCap);
    out.resize(step_nops);
    std::vector<unsigned long long> pc(4ull * kPieceCap);
    SM_CUDA(cudaMemcpyAsync(out.data(), trace_dev_step, sizeof(TraceSlot) * step_nops, cudaMemcpyDeviceToHost,
                            stream));
    SM_CUDA(cudaMemcpyAsync(pc.data(), trace_dev_pieces, 32ull * kPieceCap, cudaMemcpyDeviceToHost, stream));
    SM_CUDA(cudaMemcpyAsync(h_err, device_error_flag(), 4, cudaMemcpyDeviceToHost, stream));
    SM_CUDA(cudaStreamSynchronize(stream));
    check_step_errors();
    cached = pos + 1;
    for (uint32_t j = 0; j < kPieceCap && pc[4 * j]; ++j) {
        out.push_back(TraceSlot{pc[4 * j], pc[4 * j + 1], pc[4 * j + 3], 1000});
        out.push_back(TraceSlot{pc[4 * j + 2], pc[4 * j + 2], pc[4 * j + 2], 1001});
    }
}

uint32_t Model::step_launch_count() const {
    if (step_on) return 1;
    uint32_t n = 1 + 1 + 1;  // embed, lm_head, finalize
    for (const LayerW& L : layers) n += L.fused_v ? 5 : 6;  // QKV [+ V], attention, O, gate/up, down
    return n + (tp_size > 1 ? 1 : 0);  // the argmax all-gather
}

// After a step whose bounded waits gave up: clear the barrier, the abort
// flag and the attention tickets so the next step starts clean.
void Model::reset_step_state() {
    if (!step_bar) return;
    SM_CUDA(cudaMemsetAsync(step_bar, 0, 64, stream));
    SM_CUDA(cudaMemsetAsync(step_tickets, 0, 4ull * std::max(1u, nkv_l), stream));
}

}  // namespace smallm
