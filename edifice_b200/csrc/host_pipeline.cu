// host_pipeline.cu -- forward + backward of the diagonal scans (linear scan,
// MinGRU), of the Mamba selective scan, of attention (flash, FoX, LASER) and of
// the delta rule (DeltaNet, GatedDeltaNet) over
// HOST-resident tensors: batch rows (attention: (batch, kv head) units) are streamed through a small ring of device slots so that the
// host->device copies of chunk i+1, the kernels of chunk i and the
// device->host copies of chunk i-1 run at the same time (the two copy
// directions use separate copy engines; PCIe is full duplex).
//
// Every op here is independent per batch row, so a chunk of rows is a complete
// sub-problem and the results equal those of one whole-batch call.  Ordering:
// the helper streams first wait for everything already queued on the caller's
// stream, and the caller's stream finally waits for both helper streams (on
// every exit path once a copy was queued, errors included), so the call behaves
// like any other stream-ordered entry point: once the caller's stream has
// passed the call, no copy into or out of the caller's host buffers is pending.
#include <cstdint>

#include "edb_common.cuh"

namespace {

constexpr int kSlots = 3;  // device slots in the ring
constexpr size_t kChunkTarget = 16u << 20;  // aim for ~16 MiB per tensor per chunk

enum { HOST_LINEAR = 0, HOST_MINGRU = 1 };

size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

// Rows per chunk: about `target` bytes per [rows, L, H] tensor, but at least ~4
// chunks in flight when the batch allows it.
int chunk_rows(int B, size_t row_bytes, size_t target) {
    size_t r = row_bytes >= target ? 1 : target / row_bytes;
    const size_t quarter = ((size_t)B + 3) / 4;
    if (r > quarter) r = quarter;
    if (r < 1) r = 1;
    return (int)r;
}

int chunk_rows(int B, int L, int H, int esize) {
    return chunk_rows(B, (size_t)L * H * esize, kChunkTarget);
}

// One slot: x0, x1, dy, h, g0, g1 ([rows, L, H]) then h0, gh0 ([rows, H]).
size_t slot_bytes(int rows, int L, int H, int esize) {
    const size_t t = a256((size_t)rows * L * H * esize);
    const size_t s = a256((size_t)rows * H * esize);
    return 6 * t + 2 * s;
}

int check_shape(int dtype, int B, int L, int H) {
    if (dtype != EDB_F32 && dtype != EDB_BF16) return EDB_ERR_BAD_DTYPE;
    if (B <= 0 || L <= 0 || H <= 0) return EDB_ERR_BAD_SHAPE;
    if ((long long)B * L > 0x7fffffffLL) return EDB_ERR_BAD_SHAPE;
    return EDB_OK;
}

struct Res {
    cudaStream_t sin = nullptr, sout = nullptr;
    cudaEvent_t start = nullptr, done_in = nullptr, done = nullptr;
    cudaEvent_t in_fwd[kSlots] = {}, in[kSlots] = {}, fwd[kSlots] = {}, comp[kSlots] = {},
                free_[kSlots] = {};
    ~Res() {
        // destruction is deferred by the runtime until queued work completes
        if (sin) cudaStreamDestroy(sin);
        if (sout) cudaStreamDestroy(sout);
        for (cudaEvent_t e : {start, done_in, done})
            if (e) cudaEventDestroy(e);
        for (int i = 0; i < kSlots; ++i)
            for (cudaEvent_t e : {in_fwd[i], in[i], fwd[i], comp[i], free_[i]})
                if (e) cudaEventDestroy(e);
    }
    cudaError_t init() {
        cudaError_t e;
        if ((e = cudaStreamCreateWithFlags(&sin, cudaStreamNonBlocking))) return e;
        if ((e = cudaStreamCreateWithFlags(&sout, cudaStreamNonBlocking))) return e;
        for (cudaEvent_t* ev : {&start, &done_in, &done})
            if ((e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming))) return e;
        for (int i = 0; i < kSlots; ++i)
            for (cudaEvent_t* ev : {&in_fwd[i], &in[i], &fwd[i], &comp[i], &free_[i]})
                if ((e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming))) return e;
        return cudaSuccess;
    }
};

// Makes the caller's stream wait for both helper streams when it goes out of
// scope, on the success path and on every error path after the first copy was
// queued: a caller that synchronises its stream after an error status then
// knows that no copy into or out of its host buffers is still pending.
struct Join {
    Res& r;
    cudaStream_t s;
    bool armed = false;
    ~Join() {
        if (!armed) return;
        if (cudaEventRecord(r.done_in, r.sin) == cudaSuccess) cudaStreamWaitEvent(s, r.done_in, 0);
        if (cudaEventRecord(r.done, r.sout) == cudaSuccess) cudaStreamWaitEvent(s, r.done, 0);
    }
};

#define EDB_TRY(expr)                                   \
    do {                                                \
        cudaError_t e_ = (expr);                        \
        if (e_ != cudaSuccess) return edb::status_from_cuda(e_); \
    } while (0)
#define EDB_TRY_ST(expr)            \
    do {                            \
        int st_ = (expr);           \
        if (st_ != EDB_OK) return st_; \
    } while (0)

const char* hp(const void* p, size_t o) { return static_cast<const char*>(p) + o; }
char* hq(void* p, size_t o) { return static_cast<char*>(p) + o; }

// x0/x1: (a, b) for the linear scan, (z, c) for MinGRU.  g0/g1 likewise.
int run(int op, int dtype, const void* x0, const void* x1, const void* h0, const void* dy,
        void* h, void* g0, void* g1, void* gh0, int B, int L, int H, void* ws, size_t ws_bytes,
        void* stream) {
    if (int st = check_shape(dtype, B, L, H)) return st;
    if (!x0 || !x1 || !dy || !h || !g0 || !g1 || !ws) return EDB_ERR_NULL_POINTER;
    const int es = dtype == EDB_BF16 ? 2 : 4;
    const int rows = chunk_rows(B, L, H, es);
    const size_t sb = slot_bytes(rows, L, H, es);
    if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0) return EDB_ERR_MISALIGNED;
    if (ws_bytes < kSlots * sb) return EDB_ERR_WORKSPACE_TOO_SMALL;
    const size_t tb = a256((size_t)rows * L * H * es);
    const size_t hb = a256((size_t)rows * H * es);

    cudaStream_t s = (cudaStream_t)stream;
    Res r;
    EDB_TRY(r.init());
    Join join{r, s};
    EDB_TRY(cudaEventRecord(r.start, s));
    EDB_TRY(cudaStreamWaitEvent(r.sin, r.start, 0));
    EDB_TRY(cudaStreamWaitEvent(r.sout, r.start, 0));
    join.armed = true;

    const int nchunks = (B + rows - 1) / rows;
    for (int i = 0; i < nchunks; ++i) {
        const int slot = i % kSlots;
        const int r0 = i * rows, nr = B - r0 < rows ? B - r0 : rows;
        char* base = static_cast<char*>(ws) + slot * sb;
        void* dx0 = base;
        void* dx1 = base + tb;
        void* ddy = base + 2 * tb;
        void* dh = base + 3 * tb;
        void* dg0 = base + 4 * tb;
        void* dg1 = base + 5 * tb;
        void* dh0 = base + 6 * tb;
        void* dgh0 = base + 6 * tb + hb;
        const size_t off = (size_t)r0 * L * H * es, n = (size_t)nr * L * H * es;
        const size_t off0 = (size_t)r0 * H * es, n0 = (size_t)nr * H * es;

        // host -> device, once the slot's previous chunk has been copied out: the
        // forward's inputs first, so that the forward (and the copy of h back to the
        // host) can start while dy is still on its way in
        if (i >= kSlots) EDB_TRY(cudaStreamWaitEvent(r.sin, r.free_[slot], 0));
        EDB_TRY(cudaMemcpyAsync(dx0, hp(x0, off), n, cudaMemcpyHostToDevice, r.sin));
        EDB_TRY(cudaMemcpyAsync(dx1, hp(x1, off), n, cudaMemcpyHostToDevice, r.sin));
        if (h0) EDB_TRY(cudaMemcpyAsync(dh0, hp(h0, off0), n0, cudaMemcpyHostToDevice, r.sin));
        EDB_TRY(cudaEventRecord(r.in_fwd[slot], r.sin));
        EDB_TRY(cudaMemcpyAsync(ddy, hp(dy, off), n, cudaMemcpyHostToDevice, r.sin));
        EDB_TRY(cudaEventRecord(r.in[slot], r.sin));

        // forward, then backward, of the chunk on the caller's stream
        const void* ph0 = h0 ? dh0 : nullptr;
        void* pgh0 = gh0 ? dgh0 : nullptr;
        EDB_TRY(cudaStreamWaitEvent(s, r.in_fwd[slot], 0));
        if (op == HOST_LINEAR)
            EDB_TRY_ST(edb_linear_scan_fwd(dtype, dx0, dx1, ph0, dh, nr, L, H, s));
        else
            EDB_TRY_ST(edb_mingru_fwd(dtype, dx0, dx1, ph0, dh, nr, L, H, s));
        EDB_TRY(cudaEventRecord(r.fwd[slot], s));
        EDB_TRY(cudaStreamWaitEvent(s, r.in[slot], 0));
        if (op == HOST_LINEAR)
            EDB_TRY_ST(edb_linear_scan_bwd(dtype, dx0, ph0, dh, ddy, dg0, dg1, pgh0, nr, L, H, s));
        else
            EDB_TRY_ST(edb_mingru_bwd(dtype, dx0, dx1, ph0, dh, ddy, dg0, dg1, pgh0, nr, L, H, s));
        EDB_TRY(cudaEventRecord(r.comp[slot], s));

        // device -> host: h as soon as the forward is done, the gradients after the
        // backward (the backward only reads h, so both may run at once)
        EDB_TRY(cudaStreamWaitEvent(r.sout, r.fwd[slot], 0));
        EDB_TRY(cudaMemcpyAsync(hq(h, off), dh, n, cudaMemcpyDeviceToHost, r.sout));
        EDB_TRY(cudaStreamWaitEvent(r.sout, r.comp[slot], 0));
        EDB_TRY(cudaMemcpyAsync(hq(g0, off), dg0, n, cudaMemcpyDeviceToHost, r.sout));
        EDB_TRY(cudaMemcpyAsync(hq(g1, off), dg1, n, cudaMemcpyDeviceToHost, r.sout));
        if (gh0) EDB_TRY(cudaMemcpyAsync(hq(gh0, off0), dgh0, n0, cudaMemcpyDeviceToHost, r.sout));
        EDB_TRY(cudaEventRecord(r.free_[slot], r.sout));
    }
    return EDB_OK;  // `join` makes the caller's stream wait for the last copies
}

// ------------------------------------------------------------ selective scan
// A chunk of the selective scan is far more work per byte than a diagonal-scan
// chunk and its kernels want many rows at once (32 CTAs per row at d_inner =
// 4096), so its chunks aim at ~256 MiB per [rows, L, D] tensor.
constexpr size_t kSsmChunkTarget = 256u << 20;

struct SsmSlot {
    // [rows,L,D] io, [rows,L,N] io, [rows,L,N] f32, ckpt, bwd ws, dt mean [rows,L] f32
    // (model semantics)
    size_t td, tn, tf, ck, ws, dm;
    size_t bytes() const { return 6 * td + 2 * tn + 2 * tf + ck + ws + dm; }
};

int ssm_rows(int B, int L, int D, int es) {
    return chunk_rows(B, (size_t)L * D * es, kSsmChunkTarget);
}

SsmSlot ssm_slot(int rows, int L, int D, int N, int es, bool model = false) {
    SsmSlot g;
    g.dm = model ? a256((size_t)rows * L * 4) : 0;
    g.td = a256((size_t)rows * L * D * es);
    g.tn = a256((size_t)rows * L * N * es);
    g.tf = a256((size_t)rows * L * N * 4);
    g.ck = a256(edb_selective_scan_ckpt_bytes(rows, L, D, N));
    g.ws = a256(edb_selective_scan_bwd_workspace(rows, L, D, N, 1));
    return g;
}

int check_ssm(int dtype, int B, int L, int D, int N) {
    if (dtype != EDB_F32 && dtype != EDB_BF16) return EDB_ERR_BAD_DTYPE;
    if (B <= 0 || L <= 0 || D <= 0 || N <= 0 || N > 16) return EDB_ERR_BAD_SHAPE;
    if ((long long)B * L > 0x7fffffffLL) return EDB_ERR_BAD_SHAPE;
    return EDB_OK;
}

// model: the model semantics (edb_selective_scan_model_*); A may then be NULL (the
// fixed -(n+1) diagonal).
int run_ssm(bool model, int dtype, const void* x, const void* dt, const void* A,
            const void* Bm, const void* Cm, const void* dy, void* y, void* gx, void* gdt,
            float* gB, float* gC, int B, int L, int D, int N, float dt_min, float dt_max,
            void* ws, size_t ws_bytes, void* stream) {
    if (int st = check_ssm(dtype, B, L, D, N)) return st;
    if (!x || !dt || (!A && !model) || !Bm || !Cm || !dy || !y || !gx || !gdt || !gB || !gC ||
        !ws)
        return EDB_ERR_NULL_POINTER;
    const int es = dtype == EDB_BF16 ? 2 : 4;
    const int rows = ssm_rows(B, L, D, es);
    const SsmSlot g = ssm_slot(rows, L, D, N, es, model);
    const size_t ab = a256((size_t)D * N * es);
    if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0) return EDB_ERR_MISALIGNED;
    if (ws_bytes < ab + kSlots * g.bytes()) return EDB_ERR_WORKSPACE_TOO_SMALL;

    cudaStream_t s = (cudaStream_t)stream;
    Res r;
    EDB_TRY(r.init());
    Join join{r, s};
    EDB_TRY(cudaEventRecord(r.start, s));
    EDB_TRY(cudaStreamWaitEvent(r.sin, r.start, 0));
    EDB_TRY(cudaStreamWaitEvent(r.sout, r.start, 0));
    join.armed = true;

    // A [D, N] is shared by every row: one copy ahead of the first chunk
    void* dA = A ? ws : nullptr;
    if (A) EDB_TRY(cudaMemcpyAsync(dA, A, (size_t)D * N * es, cudaMemcpyHostToDevice, r.sin));

    const int nchunks = (B + rows - 1) / rows;
    for (int i = 0; i < nchunks; ++i) {
        const int slot = i % kSlots;
        const int r0 = i * rows, nr = B - r0 < rows ? B - r0 : rows;
        char* p = static_cast<char*>(ws) + ab + slot * g.bytes();
        void* dx = p;
        void* ddt = p + g.td;
        void* ddy = p + 2 * g.td;
        void* dyo = p + 3 * g.td;
        void* dgx = p + 4 * g.td;
        void* dgdt = p + 5 * g.td;
        void* dB = p + 6 * g.td;
        void* dC = p + 6 * g.td + g.tn;
        float* dgB = reinterpret_cast<float*>(p + 6 * g.td + 2 * g.tn);
        float* dgC = reinterpret_cast<float*>(p + 6 * g.td + 2 * g.tn + g.tf);
        float* dck = reinterpret_cast<float*>(p + 6 * g.td + 2 * g.tn + 2 * g.tf);
        void* dws = p + 6 * g.td + 2 * g.tn + 2 * g.tf + g.ck;
        float* ddm = reinterpret_cast<float*>(p + 6 * g.td + 2 * g.tn + 2 * g.tf + g.ck + g.ws);
        const size_t offd = (size_t)r0 * L * D * es, nd = (size_t)nr * L * D * es;
        const size_t offn = (size_t)r0 * L * N * es, nn = (size_t)nr * L * N * es;
        const size_t offf = (size_t)r0 * L * N, nf = (size_t)nr * L * N * 4;

        // host -> device once the slot's previous chunk has left: the forward's
        // inputs first, dY after them
        if (i >= kSlots) EDB_TRY(cudaStreamWaitEvent(r.sin, r.free_[slot], 0));
        EDB_TRY(cudaMemcpyAsync(dx, hp(x, offd), nd, cudaMemcpyHostToDevice, r.sin));
        EDB_TRY(cudaMemcpyAsync(ddt, hp(dt, offd), nd, cudaMemcpyHostToDevice, r.sin));
        EDB_TRY(cudaMemcpyAsync(dB, hp(Bm, offn), nn, cudaMemcpyHostToDevice, r.sin));
        EDB_TRY(cudaMemcpyAsync(dC, hp(Cm, offn), nn, cudaMemcpyHostToDevice, r.sin));
        EDB_TRY(cudaEventRecord(r.in_fwd[slot], r.sin));
        EDB_TRY(cudaMemcpyAsync(ddy, hp(dy, offd), nd, cudaMemcpyHostToDevice, r.sin));
        EDB_TRY(cudaEventRecord(r.in[slot], r.sin));

        // forward (writing the chunk-start states), then backward, on the caller's stream
        EDB_TRY(cudaStreamWaitEvent(s, r.in_fwd[slot], 0));
        if (model)
            EDB_TRY_ST(edb_selective_scan_model_fwd(dtype, dx, ddt, dA, dB, dC, dyo, ddm, dck, nr,
                                                    L, D, N, dt_min, dt_max, s));
        else
            EDB_TRY_ST(edb_selective_scan_fwd(dtype, dx, ddt, dA, dB, dC, dyo, dck, nr, L, D, N,
                                              dt_min, dt_max, s));
        EDB_TRY(cudaEventRecord(r.fwd[slot], s));
        EDB_TRY(cudaStreamWaitEvent(s, r.in[slot], 0));
        if (model)
            EDB_TRY_ST(edb_selective_scan_model_bwd(dtype, dx, ddt, dA, dB, dC, ddy, ddm, dck, dgx,
                                                    dgdt, dgB, dgC, nr, L, D, N, dt_min, dt_max,
                                                    dws, g.ws, s));
        else
            EDB_TRY_ST(edb_selective_scan_bwd(dtype, dx, ddt, dA, dB, dC, ddy, dck, dgx, dgdt,
                                              dgB, dgC, nr, L, D, N, dt_min, dt_max, dws, g.ws,
                                              s));
        EDB_TRY(cudaEventRecord(r.comp[slot], s));

        // device -> host: y as soon as the forward is done, the gradients after
        // the backward
        EDB_TRY(cudaStreamWaitEvent(r.sout, r.fwd[slot], 0));
        EDB_TRY(cudaMemcpyAsync(hq(y, offd), dyo, nd, cudaMemcpyDeviceToHost, r.sout));
        EDB_TRY(cudaStreamWaitEvent(r.sout, r.comp[slot], 0));
        EDB_TRY(cudaMemcpyAsync(hq(gx, offd), dgx, nd, cudaMemcpyDeviceToHost, r.sout));
        EDB_TRY(cudaMemcpyAsync(hq(gdt, offd), dgdt, nd, cudaMemcpyDeviceToHost, r.sout));
        EDB_TRY(cudaMemcpyAsync(gB + offf, dgB, nf, cudaMemcpyDeviceToHost, r.sout));
        EDB_TRY(cudaMemcpyAsync(gC + offf, dgC, nf, cudaMemcpyDeviceToHost, r.sout));
        EDB_TRY(cudaEventRecord(r.free_[slot], r.sout));
    }
    return EDB_OK;  // `join` makes the caller's stream wait for the last copies
}

// ------------------------------------------------------------ attention
// Units are (batch, kv head) pairs: unit u = b * Hkv + hk owns q / o / dO / dq
// heads [u G, u G + G) (G = Hq / Hkv; FoX's cs / dcs rows likewise) and k / v /
// dk / dv head u, contiguous in the [B, H, L, d] layouts, so a run of consecutive
// units is a complete sub-problem that the device kernels take as `batch = units,
// kv_heads = 1, q_heads = G` (LASER's v_max is per (b, kv head, column), so per
// unit too).  About eight chunks per call: copies dominate at these sizes, and
// each chunk's backward grid still covers several waves.
enum { ATTN_FLASH = 0, ATTN_FOX = 1, ATTN_LASER = 2 };

struct AttnSlot {
    // [units, G, L, d] io, [units, L, d] io, lse f32 (flash, FoX), cs and dcs f32
    // (FoX), the forward's residual (LASER), the backward's workspace
    size_t tq, tk, lse, cs, resid, ws;
    size_t bytes() const { return 4 * tq + 4 * tk + lse + 2 * cs + resid + ws; }
};

int attn_units_per_chunk(int units) { return units < 8 ? 1 : (units + 7) / 8; }

AttnSlot attn_slot(int op, int dtype, int nu, int G, int L, int d) {
    const int es = dtype == EDB_BF16 ? 2 : 4;
    AttnSlot g{};
    g.tq = a256((size_t)nu * G * L * d * es);
    g.tk = a256((size_t)nu * L * d * es);
    const size_t rows = a256((size_t)nu * G * L * 4);
    if (op != ATTN_LASER) g.lse = rows;
    if (op == ATTN_FOX) g.cs = rows;
    if (op == ATTN_LASER) g.resid = a256(edb_laser_attention_resid_bytes(dtype, nu, G, 1, L, d));
    g.ws = a256(op == ATTN_FLASH ? edb_flash_attention_bwd_workspace(dtype, nu, G, 1, L, d, 1)
                : op == ATTN_FOX ? edb_fox_attention_bwd_workspace(dtype, nu, G, 1, L, d)
                                 : edb_laser_attention_bwd_workspace(dtype, nu, G, 1, L, d));
    return g;
}

int check_attn(int dtype, int B, int Hq, int Hkv, int L, int d) {
    if (dtype != EDB_F32 && dtype != EDB_BF16) return EDB_ERR_BAD_DTYPE;
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || L <= 0 || d <= 0 || Hq % Hkv != 0)
        return EDB_ERR_BAD_SHAPE;
    return EDB_OK;
}

size_t attn_workspace(int op, int dtype, int B, int Hq, int Hkv, int L, int d) {
    if (check_attn(dtype, B, Hq, Hkv, L, d) != EDB_OK) return 0;
    return kSlots * attn_slot(op, dtype, attn_units_per_chunk(B * Hkv), Hq / Hkv, L, d).bytes();
}

// cs / dcs: FoX only (f32 [B, Hq, L]).
int run_attn(int op, int dtype, const void* q, const void* k, const void* v, const float* cs,
             const void* dO, void* o, void* dq, void* dk, void* dv, float* dcs, int B, int Hq,
             int Hkv, int L, int d, int causal, float scale, void* ws, size_t ws_bytes,
             void* stream) {
    if (int st = check_attn(dtype, B, Hq, Hkv, L, d)) return st;
    if (!q || !k || !v || !dO || !o || !dq || !dk || !dv || !ws) return EDB_ERR_NULL_POINTER;
    if (op == ATTN_FOX && (!cs || !dcs)) return EDB_ERR_NULL_POINTER;
    const int es = dtype == EDB_BF16 ? 2 : 4;
    const int G = Hq / Hkv, units = B * Hkv;
    const int nu = attn_units_per_chunk(units);
    const AttnSlot g = attn_slot(op, dtype, nu, G, L, d);
    if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0) return EDB_ERR_MISALIGNED;
    if (ws_bytes < kSlots * g.bytes()) return EDB_ERR_WORKSPACE_TOO_SMALL;

    cudaStream_t s = (cudaStream_t)stream;
    Res r;
    EDB_TRY(r.init());
    Join join{r, s};
    EDB_TRY(cudaEventRecord(r.start, s));
    EDB_TRY(cudaStreamWaitEvent(r.sin, r.start, 0));
    EDB_TRY(cudaStreamWaitEvent(r.sout, r.start, 0));
    join.armed = true;

    const int nchunks = (units + nu - 1) / nu;
    for (int i = 0; i < nchunks; ++i) {
        const int slot = i % kSlots;
        const int u0 = i * nu, n = units - u0 < nu ? units - u0 : nu;
        char* p = static_cast<char*>(ws) + slot * g.bytes();
        void* dqi = p;
        void* ddo = p + g.tq;
        void* dout = p + 2 * g.tq;
        void* ddq = p + 3 * g.tq;
        char* pk = p + 4 * g.tq;
        void* dki = pk;
        void* dvi = pk + g.tk;
        void* ddk = pk + 2 * g.tk;
        void* ddv = pk + 3 * g.tk;
        char* pr = pk + 4 * g.tk;
        float* dlse = reinterpret_cast<float*>(pr);
        float* dcsi = reinterpret_cast<float*>(pr + g.lse);
        float* ddcs = reinterpret_cast<float*>(pr + g.lse + g.cs);
        void* dres = pr + g.lse + 2 * g.cs;
        void* dws = pr + g.lse + 2 * g.cs + g.resid;
        const size_t offq = (size_t)u0 * G * L * d * es, nq = (size_t)n * G * L * d * es;
        const size_t offk = (size_t)u0 * L * d * es, nk = (size_t)n * L * d * es;
        const size_t offr = (size_t)u0 * G * L, nr = (size_t)n * G * L * 4;

        // host -> device once the slot's previous chunk has left: the forward's
        // inputs, then dO
        if (i >= kSlots) EDB_TRY(cudaStreamWaitEvent(r.sin, r.free_[slot], 0));
        EDB_TRY(cudaMemcpyAsync(dqi, hp(q, offq), nq, cudaMemcpyHostToDevice, r.sin));
        EDB_TRY(cudaMemcpyAsync(dki, hp(k, offk), nk, cudaMemcpyHostToDevice, r.sin));
        EDB_TRY(cudaMemcpyAsync(dvi, hp(v, offk), nk, cudaMemcpyHostToDevice, r.sin));
        if (op == ATTN_FOX)
            EDB_TRY(cudaMemcpyAsync(dcsi, cs + offr, nr, cudaMemcpyHostToDevice, r.sin));
        EDB_TRY(cudaEventRecord(r.in_fwd[slot], r.sin));
        EDB_TRY(cudaMemcpyAsync(ddo, hp(dO, offq), nq, cudaMemcpyHostToDevice, r.sin));
        EDB_TRY(cudaEventRecord(r.in[slot], r.sin));

        // forward, then backward, on the caller's stream
        EDB_TRY(cudaStreamWaitEvent(s, r.in_fwd[slot], 0));
        if (op == ATTN_FLASH)
            EDB_TRY_ST(edb_flash_attention_fwd(dtype, dqi, dki, dvi, dout, dlse, n, G, 1, L, d,
                                               causal, scale, s));
        else if (op == ATTN_FOX)
            EDB_TRY_ST(edb_fox_attention_fwd(dtype, dqi, dki, dvi, dcsi, dout, dlse, n, G, 1, L,
                                             d, scale, s));
        else
            EDB_TRY_ST(edb_laser_attention_fwd(dtype, dqi, dki, dvi, nullptr, dout, dres, n, G,
                                               1, L, d, causal, scale, s));
        EDB_TRY(cudaEventRecord(r.fwd[slot], s));
        EDB_TRY(cudaStreamWaitEvent(s, r.in[slot], 0));
        if (op == ATTN_FLASH)
            EDB_TRY_ST(edb_flash_attention_bwd(dtype, dqi, dki, dvi, dout, ddo, dlse, ddq, ddk,
                                               ddv, n, G, 1, L, d, causal, scale, dws, g.ws, s));
        else if (op == ATTN_FOX)
            EDB_TRY_ST(edb_fox_attention_bwd(dtype, dqi, dki, dvi, dcsi, dout, ddo, dlse, ddq,
                                             ddk, ddv, ddcs, n, G, 1, L, d, scale, dws, g.ws, s));
        else
            EDB_TRY_ST(edb_laser_attention_bwd(dtype, dqi, dki, ddo, dres, ddq, ddk, ddv, n, G,
                                               1, L, d, causal, scale, dws, g.ws, s));
        EDB_TRY(cudaEventRecord(r.comp[slot], s));

        // device -> host: o as soon as the forward is done, the gradients after the
        // backward
        EDB_TRY(cudaStreamWaitEvent(r.sout, r.fwd[slot], 0));
        EDB_TRY(cudaMemcpyAsync(hq(o, offq), dout, nq, cudaMemcpyDeviceToHost, r.sout));
        EDB_TRY(cudaStreamWaitEvent(r.sout, r.comp[slot], 0));
        EDB_TRY(cudaMemcpyAsync(hq(dq, offq), ddq, nq, cudaMemcpyDeviceToHost, r.sout));
        EDB_TRY(cudaMemcpyAsync(hq(dk, offk), ddk, nk, cudaMemcpyDeviceToHost, r.sout));
        EDB_TRY(cudaMemcpyAsync(hq(dv, offk), ddv, nk, cudaMemcpyDeviceToHost, r.sout));
        if (op == ATTN_FOX)
            EDB_TRY(cudaMemcpyAsync(dcs + offr, ddcs, nr, cudaMemcpyDeviceToHost, r.sout));
        EDB_TRY(cudaEventRecord(r.free_[slot], r.sout));
    }
    return EDB_OK;  // `join` makes the caller's stream wait for the last copies
}

// ------------------------------------------------------------ delta rule
// DeltaNet / GatedDeltaNet: every [B, L, H, ...] tensor is contiguous per batch row
// and a row's (b, h) recurrences are complete sub-problems, so chunks of rows go
// through the same ring.  Each slot runs its chunk's kernels on a compute stream of
// its own: a chunk's state passes (chunked form) or token recurrence (the other
// forms) are serial chains over the sequence that occupy a fraction of the GPU,
// so consecutive chunks' kernels overlap instead of queueing behind each other.
size_t delta_row_elems(int L, int H, int d) { return (size_t)L * H * d; }

struct DeltaSlot {
    // [rows, L, H, d] io (q, k, v, dO, o, dq, dk, dv), beta and its gradient,
    // alpha and its gradient (gated), the forward's residual, the scratch of the
    // forward and of the backward (one after the other on the slot's stream)
    size_t t, tb, ta, resid, ws;
    size_t bytes() const { return 8 * t + 2 * tb + 2 * ta + resid + ws; }
};

// Whether the call takes the chunked tensor-core form (a forward workspace) or the
// token recurrence.
bool delta_chunked(bool gated, int dtype, int bpe, int L, int H, int d) {
    return (gated ? edb_gated_delta_net_fwd_workspace(dtype, bpe, 1, L, H, d)
                  : edb_delta_rule_fwd_workspace(dtype, bpe, 1, L, H, d)) > 0;
}

// The token recurrence's chunks are long serial chains (each about as long as the
// whole batch's), so it takes at most one chunk per slot, all in flight at once;
// the chunked form's chunks are short next to their copies.
int delta_rows(bool gated, int dtype, int bpe, int B, int L, int H, int d) {
    const int es = dtype == EDB_BF16 ? 2 : 4;
    if (!delta_chunked(gated, dtype, bpe, L, H, d)) return (B + kSlots - 1) / kSlots;
    return chunk_rows(B, delta_row_elems(L, H, d) * es, 64u << 20);
}

DeltaSlot delta_slot(bool gated, int dtype, int bpe, int rows, int L, int H, int d) {
    const int es = dtype == EDB_BF16 ? 2 : 4;
    DeltaSlot g{};
    g.t = a256((size_t)rows * delta_row_elems(L, H, d) * es);
    g.tb = a256((size_t)rows * L * H * (bpe ? d : 1) * es);
    g.ta = gated ? a256((size_t)rows * L * H * es) : 0;
    size_t fw, bw;
    if (gated) {
        g.resid = a256(edb_gated_delta_net_ckpt_bytes(dtype, bpe, rows, L, H, d));
        fw = edb_gated_delta_net_fwd_workspace(dtype, bpe, rows, L, H, d);
        bw = edb_gated_delta_net_bwd_workspace(dtype, bpe, rows, L, H, d, 1);
    } else {
        g.resid = a256(edb_delta_rule_ckpt_bytes(dtype, bpe, rows, L, H, d));
        fw = edb_delta_rule_fwd_workspace(dtype, bpe, rows, L, H, d);
        bw = edb_delta_rule_bwd_workspace(dtype, bpe, rows, L, H, d, 1);
    }
    g.ws = a256(fw > bw ? fw : bw);
    return g;
}

int check_delta(int dtype, int B, int L, int H, int d) {
    if (dtype != EDB_F32 && dtype != EDB_BF16) return EDB_ERR_BAD_DTYPE;
    if (B <= 0 || L <= 0 || H <= 0 || d <= 0 || d > 128) return EDB_ERR_BAD_SHAPE;
    return EDB_OK;
}

size_t delta_workspace(bool gated, int dtype, int bpe, int B, int L, int H, int d) {
    if (check_delta(dtype, B, L, H, d) != EDB_OK) return 0;
    return kSlots * delta_slot(gated, dtype, bpe, delta_rows(gated, dtype, bpe, B, L, H, d), L,
                               H, d).bytes();
}

// The slots' compute streams, joined into the caller's stream on every exit path
// once work was queued on them.
struct SlotStreams {
    cudaStream_t cs[kSlots] = {};
    cudaEvent_t done[kSlots] = {};
    cudaStream_t s = nullptr;
    bool armed = false;
    cudaError_t init(cudaStream_t caller) {
        s = caller;
        cudaError_t e;
        for (int i = 0; i < kSlots; ++i) {
            if ((e = cudaStreamCreateWithFlags(&cs[i], cudaStreamNonBlocking))) return e;
            if ((e = cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming))) return e;
        }
        return cudaSuccess;
    }
    ~SlotStreams() {
        for (int i = 0; i < kSlots; ++i) {
            if (armed && cs[i] && done[i] && cudaEventRecord(done[i], cs[i]) == cudaSuccess)
                cudaStreamWaitEvent(s, done[i], 0);
            if (cs[i]) cudaStreamDestroy(cs[i]);
            if (done[i]) cudaEventDestroy(done[i]);
        }
    }
};

// alpha / galpha: GatedDeltaNet when alpha is not null.
int run_delta(int dtype, const void* q, const void* k, const void* v, const void* beta,
              int bpe, const void* alpha, const void* dO, void* o, void* gq, void* gk, void* gv,
              void* gbeta, void* galpha, int B, int L, int H, int d, void* ws, size_t ws_bytes,
              void* stream) {
    if (int st = check_delta(dtype, B, L, H, d)) return st;
    const bool gated = alpha != nullptr;
    if (!q || !k || !v || !beta || !dO || !o || !gq || !gk || !gv || !gbeta || !ws ||
        (gated && !galpha))
        return EDB_ERR_NULL_POINTER;
    const int es = dtype == EDB_BF16 ? 2 : 4;
    const int rows = delta_rows(gated, dtype, bpe, B, L, H, d);
    const DeltaSlot g = delta_slot(gated, dtype, bpe, rows, L, H, d);
    if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0) return EDB_ERR_MISALIGNED;
    if (ws_bytes < kSlots * g.bytes()) return EDB_ERR_WORKSPACE_TOO_SMALL;

    cudaStream_t s = (cudaStream_t)stream;
    Res r;
    EDB_TRY(r.init());
    SlotStreams ss;
    EDB_TRY(ss.init(s));
    Join join{r, s};
    EDB_TRY(cudaEventRecord(r.start, s));
    EDB_TRY(cudaStreamWaitEvent(r.sin, r.start, 0));
    EDB_TRY(cudaStreamWaitEvent(r.sout, r.start, 0));
    for (int i = 0; i < kSlots; ++i) EDB_TRY(cudaStreamWaitEvent(ss.cs[i], r.start, 0));
    join.armed = true;
    ss.armed = true;

    const int nchunks = (B + rows - 1) / rows;
    for (int i = 0; i < nchunks; ++i) {
        const int slot = i % kSlots;
        cudaStream_t c = ss.cs[slot];
        const int r0 = i * rows, nr = B - r0 < rows ? B - r0 : rows;
        char* p = static_cast<char*>(ws) + slot * g.bytes();
        void* dq_ = p;
        void* dk_ = p + g.t;
        void* dv_ = p + 2 * g.t;
        void* ddo = p + 3 * g.t;
        void* dout = p + 4 * g.t;
        void* dgq = p + 5 * g.t;
        void* dgk = p + 6 * g.t;
        void* dgv = p + 7 * g.t;
        void* dbeta = p + 8 * g.t;
        void* dgbeta = p + 8 * g.t + g.tb;
        void* dalpha = p + 8 * g.t + 2 * g.tb;
        void* dgalpha = p + 8 * g.t + 2 * g.tb + g.ta;
        float* dres = reinterpret_cast<float*>(p + 8 * g.t + 2 * g.tb + 2 * g.ta);
        void* dws = p + 8 * g.t + 2 * g.tb + 2 * g.ta + g.resid;
        const size_t row_t = delta_row_elems(L, H, d) * es;
        const size_t row_b = (size_t)L * H * (bpe ? d : 1) * es, row_a = (size_t)L * H * es;
        const size_t ot = r0 * row_t, nt = nr * row_t;
        const size_t ob = r0 * row_b, nb = nr * row_b, oa = r0 * row_a, na = nr * row_a;

        // host -> device once the slot's previous chunk has left: the forward's
        // inputs, then dO
        if (i >= kSlots) EDB_TRY(cudaStreamWaitEvent(r.sin, r.free_[slot], 0));
        EDB_TRY(cudaMemcpyAsync(dq_, hp(q, ot), nt, cudaMemcpyHostToDevice, r.sin));
        EDB_TRY(cudaMemcpyAsync(dk_, hp(k, ot), nt, cudaMemcpyHostToDevice, r.sin));
        EDB_TRY(cudaMemcpyAsync(dv_, hp(v, ot), nt, cudaMemcpyHostToDevice, r.sin));
        EDB_TRY(cudaMemcpyAsync(dbeta, hp(beta, ob), nb, cudaMemcpyHostToDevice, r.sin));
        if (gated)
            EDB_TRY(cudaMemcpyAsync(dalpha, hp(alpha, oa), na, cudaMemcpyHostToDevice, r.sin));
        EDB_TRY(cudaEventRecord(r.in_fwd[slot], r.sin));
        EDB_TRY(cudaMemcpyAsync(ddo, hp(dO, ot), nt, cudaMemcpyHostToDevice, r.sin));
        EDB_TRY(cudaEventRecord(r.in[slot], r.sin));

        // forward (leaving its residual), then backward, on the slot's stream
        EDB_TRY(cudaStreamWaitEvent(c, r.in_fwd[slot], 0));
        if (gated)
            EDB_TRY_ST(edb_gated_delta_net_fwd_ws(dtype, dq_, dk_, dv_, dbeta, bpe, dalpha, dout,
                                                  dres, nr, L, H, d, dws, g.ws, c));
        else
            EDB_TRY_ST(edb_delta_rule_fwd(dtype, dq_, dk_, dv_, dbeta, bpe, dout, dres, nr, L, H,
                                          d, dws, g.ws, c));
        EDB_TRY(cudaEventRecord(r.fwd[slot], c));
        EDB_TRY(cudaStreamWaitEvent(c, r.in[slot], 0));
        if (gated)
            EDB_TRY_ST(edb_gated_delta_net_bwd(dtype, dq_, dk_, dv_, dbeta, bpe, dalpha, ddo, dres,
                                               dgq, dgk, dgv, dgbeta, dgalpha, nr, L, H, d, dws,
                                               g.ws, c));
        else
            EDB_TRY_ST(edb_delta_rule_bwd(dtype, dq_, dk_, dv_, dbeta, bpe, ddo, dres, dgq, dgk,
                                          dgv, dgbeta, nr, L, H, d, dws, g.ws, c));
        EDB_TRY(cudaEventRecord(r.comp[slot], c));

        // device -> host: o once the forward is done, the gradients after the backward
        EDB_TRY(cudaStreamWaitEvent(r.sout, r.fwd[slot], 0));
        EDB_TRY(cudaMemcpyAsync(hq(o, ot), dout, nt, cudaMemcpyDeviceToHost, r.sout));
        EDB_TRY(cudaStreamWaitEvent(r.sout, r.comp[slot], 0));
        EDB_TRY(cudaMemcpyAsync(hq(gq, ot), dgq, nt, cudaMemcpyDeviceToHost, r.sout));
        EDB_TRY(cudaMemcpyAsync(hq(gk, ot), dgk, nt, cudaMemcpyDeviceToHost, r.sout));
        EDB_TRY(cudaMemcpyAsync(hq(gv, ot), dgv, nt, cudaMemcpyDeviceToHost, r.sout));
        EDB_TRY(cudaMemcpyAsync(hq(gbeta, ob), dgbeta, nb, cudaMemcpyDeviceToHost, r.sout));
        if (gated)
            EDB_TRY(cudaMemcpyAsync(hq(galpha, oa), dgalpha, na, cudaMemcpyDeviceToHost, r.sout));
        EDB_TRY(cudaEventRecord(r.free_[slot], r.sout));
    }
    return EDB_OK;  // `ss` and `join` make the caller's stream wait for the rest
}

}  // namespace

extern "C" size_t edb_delta_rule_train_host_workspace(int dtype, int beta_per_element,
                                                      int batch, int seq_len, int heads,
                                                      int head_dim) {
    return delta_workspace(false, dtype, beta_per_element, batch, seq_len, heads, head_dim);
}

extern "C" int edb_delta_rule_train_host(int dtype, const void* q, const void* k, const void* v,
                                         const void* beta, int beta_per_element,
                                         const void* dO, void* o, void* gq, void* gk, void* gv,
                                         void* gbeta, int batch, int seq_len, int heads,
                                         int head_dim, void* workspace, size_t workspace_bytes,
                                         void* stream) {
    return run_delta(dtype, q, k, v, beta, beta_per_element, nullptr, dO, o, gq, gk, gv, gbeta,
                     nullptr, batch, seq_len, heads, head_dim, workspace, workspace_bytes,
                     stream);
}

extern "C" size_t edb_gated_delta_net_train_host_workspace(int dtype, int beta_per_element,
                                                           int batch, int seq_len, int heads,
                                                           int head_dim) {
    return delta_workspace(true, dtype, beta_per_element, batch, seq_len, heads, head_dim);
}

extern "C" int edb_gated_delta_net_train_host(int dtype, const void* q, const void* k,
                                              const void* v, const void* beta,
                                              int beta_per_element, const void* alpha,
                                              const void* dO, void* o, void* gq, void* gk,
                                              void* gv, void* gbeta, void* galpha, int batch,
                                              int seq_len, int heads, int head_dim,
                                              void* workspace, size_t workspace_bytes,
                                              void* stream) {
    if (!alpha) return EDB_ERR_NULL_POINTER;
    return run_delta(dtype, q, k, v, beta, beta_per_element, alpha, dO, o, gq, gk, gv, gbeta,
                     galpha, batch, seq_len, heads, head_dim, workspace, workspace_bytes,
                     stream);
}

extern "C" size_t edb_flash_attention_train_host_workspace(int dtype, int batch, int q_heads,
                                                           int kv_heads, int seq_len,
                                                           int head_dim) {
    return attn_workspace(ATTN_FLASH, dtype, batch, q_heads, kv_heads, seq_len, head_dim);
}

extern "C" int edb_flash_attention_train_host(int dtype, const void* q, const void* k,
                                              const void* v, const void* dO, void* o, void* dq,
                                              void* dk, void* dv, int batch, int q_heads,
                                              int kv_heads, int seq_len, int head_dim,
                                              int causal, float scale, void* workspace,
                                              size_t workspace_bytes, void* stream) {
    return run_attn(ATTN_FLASH, dtype, q, k, v, nullptr, dO, o, dq, dk, dv, nullptr, batch,
                    q_heads, kv_heads, seq_len, head_dim, causal, scale, workspace,
                    workspace_bytes, stream);
}

extern "C" size_t edb_fox_attention_train_host_workspace(int dtype, int batch, int q_heads,
                                                         int kv_heads, int seq_len,
                                                         int head_dim) {
    return attn_workspace(ATTN_FOX, dtype, batch, q_heads, kv_heads, seq_len, head_dim);
}

extern "C" int edb_fox_attention_train_host(int dtype, const void* q, const void* k,
                                            const void* v, const float* cs, const void* dO,
                                            void* o, void* dq, void* dk, void* dv, float* dcs,
                                            int batch, int q_heads, int kv_heads, int seq_len,
                                            int head_dim, float scale, void* workspace,
                                            size_t workspace_bytes, void* stream) {
    return run_attn(ATTN_FOX, dtype, q, k, v, cs, dO, o, dq, dk, dv, dcs, batch, q_heads,
                    kv_heads, seq_len, head_dim, 1, scale, workspace, workspace_bytes, stream);
}

extern "C" size_t edb_laser_attention_train_host_workspace(int dtype, int batch, int q_heads,
                                                           int kv_heads, int seq_len,
                                                           int head_dim) {
    return attn_workspace(ATTN_LASER, dtype, batch, q_heads, kv_heads, seq_len, head_dim);
}

extern "C" int edb_laser_attention_train_host(int dtype, const void* q, const void* k,
                                              const void* v, const void* dO, void* o, void* dq,
                                              void* dk, void* dv, int batch, int q_heads,
                                              int kv_heads, int seq_len, int head_dim,
                                              int causal, float scale, void* workspace,
                                              size_t workspace_bytes, void* stream) {
    return run_attn(ATTN_LASER, dtype, q, k, v, nullptr, dO, o, dq, dk, dv, nullptr, batch,
                    q_heads, kv_heads, seq_len, head_dim, causal, scale, workspace,
                    workspace_bytes, stream);
}

extern "C" size_t edb_scan_train_host_workspace(int dtype, int batch, int seq_len, int hidden) {
    if (check_shape(dtype, batch, seq_len, hidden) != EDB_OK) return 0;
    const int es = dtype == EDB_BF16 ? 2 : 4;
    return kSlots * slot_bytes(chunk_rows(batch, seq_len, hidden, es), seq_len, hidden, es);
}

extern "C" int edb_linear_scan_train_host(int dtype, const void* a, const void* b,
                                          const void* h0, const void* dy, void* h, void* ga,
                                          void* gb, void* gh0, int batch, int seq_len,
                                          int hidden, void* workspace, size_t workspace_bytes,
                                          void* stream) {
    return run(HOST_LINEAR, dtype, a, b, h0, dy, h, ga, gb, gh0, batch, seq_len, hidden,
               workspace, workspace_bytes, stream);
}

extern "C" int edb_mingru_train_host(int dtype, const void* z, const void* c, const void* h0,
                                     const void* dy, void* h, void* gz, void* gc, void* gh0,
                                     int batch, int seq_len, int hidden, void* workspace,
                                     size_t workspace_bytes, void* stream) {
    return run(HOST_MINGRU, dtype, z, c, h0, dy, h, gz, gc, gh0, batch, seq_len, hidden,
               workspace, workspace_bytes, stream);
}

extern "C" size_t edb_selective_scan_train_host_workspace(int dtype, int batch, int seq_len,
                                                          int d_inner, int d_state) {
    if (check_ssm(dtype, batch, seq_len, d_inner, d_state) != EDB_OK) return 0;
    const int es = dtype == EDB_BF16 ? 2 : 4;
    const int rows = ssm_rows(batch, seq_len, d_inner, es);
    return a256((size_t)d_inner * d_state * es) +
           kSlots * ssm_slot(rows, seq_len, d_inner, d_state, es).bytes();
}

extern "C" int edb_selective_scan_train_host(int dtype, const void* x, const void* dt,
                                             const void* A, const void* B, const void* C,
                                             const void* dy, void* y, void* gx, void* gdt,
                                             float* gB, float* gC, int batch, int seq_len,
                                             int d_inner, int d_state, float dt_min,
                                             float dt_max, void* workspace,
                                             size_t workspace_bytes, void* stream) {
    return run_ssm(false, dtype, x, dt, A, B, C, dy, y, gx, gdt, gB, gC, batch, seq_len,
                   d_inner, d_state, dt_min, dt_max, workspace, workspace_bytes, stream);
}

extern "C" size_t edb_selective_scan_model_train_host_workspace(int dtype, int batch,
                                                                int seq_len, int d_inner,
                                                                int d_state) {
    if (check_ssm(dtype, batch, seq_len, d_inner, d_state) != EDB_OK) return 0;
    const int es = dtype == EDB_BF16 ? 2 : 4;
    const int rows = ssm_rows(batch, seq_len, d_inner, es);
    return a256((size_t)d_inner * d_state * es) +
           kSlots * ssm_slot(rows, seq_len, d_inner, d_state, es, true).bytes();
}

extern "C" int edb_selective_scan_model_train_host(int dtype, const void* x, const void* dt,
                                                   const void* A, const void* B, const void* C,
                                                   const void* dy, void* y, void* gx, void* gdt,
                                                   float* gB, float* gC, int batch, int seq_len,
                                                   int d_inner, int d_state, float dt_min,
                                                   float dt_max, void* workspace,
                                                   size_t workspace_bytes, void* stream) {
    return run_ssm(true, dtype, x, dt, A, B, C, dy, y, gx, gdt, gB, gC, batch, seq_len,
                   d_inner, d_state, dt_min, dt_max, workspace, workspace_bytes, stream);
}
