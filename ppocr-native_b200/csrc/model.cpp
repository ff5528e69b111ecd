// The CUDA backend of the ppocr-native engine: a PPOCRPL1 plan on one GPU,
// run over lanes of images (the Vulkan `GpuModel` it replaces is ppocr-native
// `src/engine/gpu/mod.rs:81-291`).
//
// Layout in device memory. Weights: every operation's weight and bias blocks
// re-packed into one arena, each block on a 256-byte boundary, so kernels may
// read them as float4. Tensors: lanes of equal size form a group that runs
// as one batch; each plan buffer of a group is one allocation of
// lanes x (the most floats any operation writes there), tensors stored NHWC
// with the lanes back to back. Scratch: per group, the f64 partial sums of
// the channel means and the per-column-block states of the CTC head.
//
// Schedule. The plan's operations are grouped into steps by `fuse`: a
// depthwise layer and the pointwise one it feeds run as one kernel; a
// squeeze-and-excite gate is folded into the next pointwise layer's input
// load; a residual add into the epilogue of the layer that produces one of
// its terms; the RSE gate and its residual add into one pass; nearest
// upsampling and channel concatenation into the sources of the dense
// convolution that reads them (the reference's own GPU fusion rules,
// gpu/mod.rs:458-533, and CPU ones, schedule.rs:273-466). Each step is a
// closure that launches its kernels on the model's stream; the whole run is
// captured once per set of sizes into a CUDA graph and replayed.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <string>
#include <thread>
#include <vector>

#include "../../include/ppocr_cuda.h"
#include "kernels.hpp"
#include "plan.hpp"

using namespace ppocr;

namespace {

thread_local std::string g_error;

int fail(int code, const std::string &msg) {
    g_error = msg;
    return code;
}

bool cuda_ok(cudaError_t e, const char *what, int *code = nullptr) {
    if (e == cudaSuccess) return true;
    g_error = std::string(what) + ": " + cudaGetErrorString(e);
    if (code) *code = e == cudaErrorMemoryAllocation ? PPOCR_E_NOMEM : PPOCR_E_DEVICE;
    return false;
}

// Tiles per CTA at least, in throughput mode (PPOCR_OPT_THROUGHPUT).
constexpr int THROUGHPUT_TILES = 4;

// Raise per-kernel limits once per device.
void configure_device(int device) {
    static std::mutex mu;
    static std::set<int> done;
    std::lock_guard<std::mutex> lock(mu);
    if (done.count(device)) return;
    configure_dw_kernels();
    configure_conv_kernels();
    configure_misc_kernels();
    configure_tc_kernels();
    done.insert(device);
}

struct DeviceBuffer {
    void *p = nullptr;
    size_t bytes = 0;
    DeviceBuffer() = default;
    DeviceBuffer(const DeviceBuffer &) = delete;
    DeviceBuffer &operator=(const DeviceBuffer &) = delete;
    ~DeviceBuffer() {
        if (p) cudaFree(p);
    }
};

struct HostBuffer {
    void *p = nullptr;
    size_t bytes = 0;
    HostBuffer() = default;
    HostBuffer(const HostBuffer &) = delete;
    HostBuffer &operator=(const HostBuffer &) = delete;
    ~HostBuffer() {
        if (p) cudaFreeHost(p);
    }
};

// Buffers of a new set of sizes take over the previous set's allocation
// when it is large enough and allocate (with a quarter of headroom) only when
// they grow, as the reference's lanes do (`gpu/mod.rs:297-388`): a run of
// new sizes then costs no cudaMalloc / cudaFree, which would synchronize the
// device, and no page-locked allocation.
bool reserve(DeviceBuffer &b, DeviceBuffer *old, size_t bytes, const char *what, int &code) {
    b.bytes = bytes;
    if (old && old->p && old->bytes >= bytes) {
        b.p = old->p;
        b.bytes = old->bytes;
        old->p = nullptr;
        return true;
    }
    const size_t grown = bytes + bytes / 4;
    if (!cuda_ok(cudaMalloc(&b.p, grown), what, &code)) return false;
    b.bytes = grown;
    return true;
}

bool reserve(HostBuffer &b, HostBuffer *old, size_t bytes, const char *what, int &code) {
    b.bytes = bytes;
    if (old && old->p && old->bytes >= bytes) {
        b.p = old->p;
        b.bytes = old->bytes;
        old->p = nullptr;
        return true;
    }
    const size_t grown = bytes + bytes / 4;
    if (!cuda_ok(cudaHostAlloc(&b.p, grown, cudaHostAllocDefault), what, &code)) return false;
    b.bytes = grown;
    return true;
}

// Weights on one device, shared by the models made with share_weights.
struct Weights {
    int device = 0;
    DeviceBuffer arena;
    std::vector<size_t> w_at, b_at;  // per op: float offset of its blocks in the arena (or SIZE_MAX)
    // Pointwise layers' weights for the tensor-core kernel: transposed to
    // [n][kpad], split into tf32 halves (SIZE_MAX: none).
    DeviceBuffer tc_arena;
    std::vector<size_t> tc_hi_at, tc_lo_at;
    std::vector<int> tc_kpad;
    std::vector<float> tc_wmax, tc_bmax;  // CTC heads: largest |w|, |b| over the live columns
    std::vector<char> tc_fold;            // the copy has its horizontal taps folded into N (TcArgs::fold)
    const float *tc_hi(size_t op) const {
        return tc_hi_at[op] == SIZE_MAX ? nullptr : static_cast<const float *>(tc_arena.p) + tc_hi_at[op];
    }
    const float *tc_lo(size_t op) const {
        return tc_lo_at[op] == SIZE_MAX ? nullptr : static_cast<const float *>(tc_arena.p) + tc_lo_at[op];
    }
    const float *w(size_t op) const {
        return w_at[op] == SIZE_MAX ? nullptr : static_cast<const float *>(arena.p) + w_at[op];
    }
    const float *b(size_t op) const {
        return b_at[op] == SIZE_MAX ? nullptr : static_cast<const float *>(arena.p) + b_at[op];
    }
};

// ------------------------------------------------------------- fusion plan

enum StepKind {
    S_OP,        // one plan operation, its own kernel(s)
    S_DW_PW,     // depthwise `a` feeding pointwise `b` [+ residual add `c`]
    S_CONV,      // a dense convolution with optional gate, sources, residual
    S_GATE_ADD,  // channelmul `a` and add `b`: y = act(x * g + x)
    S_GATE_UPADD,  // upsample-add `a` whose full-size input is the gate-add of channelmul `b` and
                   // add `c` (its only reader), computed on the fly: y = act(x2 * g + x2) + up(x)
    S_SKIP,      // folded into another step
};

struct Step {
    StepKind kind = S_OP;
    size_t op = 0;              // the operation whose output this step writes (its position)
    size_t a = 0, b = 0, c = 0; // ops involved (dw, pw, add / channelmul, add)
    bool has_add = false;       // residual add folded in (op `c`)
    bool gated = false;         // SE gate folded in: the conv reads channelmul `a`'s inputs
    // Sources of a dense conv: (buffer, channels, shift), in channel order.
    struct Src {
        size_t slot, c;
        int shift;
    };
    std::vector<Src> srcs;
    std::string name;
};

// Which later operations read the value op `i` writes, until the buffer is
// written again; `out` when that value is a plan output.
struct Uses {
    std::vector<size_t> readers;
    bool out = false;
};

std::vector<Uses> find_uses(const Plan &p) {
    std::vector<Uses> u(p.ops.size());
    for (size_t i = 0; i < p.ops.size(); i++) {
        size_t y = p.ops[i].y;
        size_t j = i + 1;
        for (; j < p.ops.size(); j++) {
            const Op &o = p.ops[j];
            if (o.x == y || (o.has_second() && o.x2 == y)) u[i].readers.push_back(j);
            if (o.y == y) break;
        }
        if (j == p.ops.size())
            for (size_t s : p.outputs)
                if (s == y) u[i].out = true;
    }
    return u;
}

bool only_reader(const Uses &u, size_t j) { return !u.out && u.readers.size() == 1 && u.readers[0] == j; }

// No op strictly between i and j writes buffer `slot`.
bool intact(const Plan &p, size_t slot, size_t i, size_t j) {
    for (size_t k = i + 1; k < j; k++)
        if (p.ops[k].y == slot) return false;
    return true;
}

bool is_pow2(size_t v, int &shift) {
    shift = 0;
    while ((size_t(1) << shift) < v) shift++;
    return (size_t(1) << shift) == v && shift < 16;
}

// The channel sources of a dense windowed conv reading a chain of
// concatenations of (nearest-upsampled) tensors; false when it is not one.
bool chain_sources(const Plan &p, const std::vector<Uses> &u, size_t conv, size_t slot, size_t before, int shift,
                   std::vector<Step::Src> &out, std::vector<size_t> &folded) {
    // The op before `before` that wrote `slot`.
    size_t w = SIZE_MAX;
    for (size_t k = before; k-- > 0;)
        if (p.ops[k].y == slot) { w = k; break; }
    if (w != SIZE_MAX && only_reader(u[w], before) && intact(p, slot, w, conv)) {
        const Op &o = p.ops[w];
        int s;
        if (o.kind == K_UPSAMPLE && o.sh == o.sw && is_pow2(o.sh, s) && s > 0 && shift + s < 16) {
            folded.push_back(w);
            return chain_sources(p, u, conv, o.x, w, shift + s, out, folded);
        }
        if (o.kind == K_CONCATC) {
            folded.push_back(w);
            return chain_sources(p, u, conv, o.x, w, shift, out, folded) &&
                   chain_sources(p, u, conv, o.x2, w, shift, out, folded);
        }
    }
    // A plain tensor: it must still hold its value when the conv runs.
    size_t c = 0;
    {
        size_t k = before;
        for (; k-- > 0;)
            if (p.ops[k].y == slot) { c = p.ops[k].oc; break; }
        if (k == SIZE_MAX) {
            if (slot != p.slot) return false;
            c = p.c;
        }
    }
    if (!intact(p, slot, before, conv)) return false;
    out.push_back({slot, c, shift});
    return out.size() <= MAX_SOURCES;
}

std::vector<Step> fuse(const Plan &p, bool enabled) {
    std::vector<Step> steps(p.ops.size());
    for (size_t i = 0; i < p.ops.size(); i++) {
        steps[i].kind = S_OP;
        steps[i].op = i;
        steps[i].a = i;
        steps[i].name = kind_name(p.ops[i].kind);
    }
    if (!enabled) return steps;
    std::vector<Uses> u = find_uses(p);
    // A fused kernel must not write a buffer it reads: the plan rules that
    // out per operation (plan.rs:680-685), not across the ones fused here.
    auto disjoint = [](const std::vector<size_t> &reads, size_t write) {
        return std::find(reads.begin(), reads.end(), write) == reads.end();
    };
    auto residual = [&](Step &st, size_t producer, size_t pos, std::vector<size_t> reads) {
        // An add right after `pos` reading the producer's output once.
        size_t j = pos + 1;
        if (j >= p.ops.size() || !only_reader(u[producer], j)) return;
        const Op &add = p.ops[j];
        if (add.kind != K_ADD || add.x == add.x2) return;
        size_t other = add.x == p.ops[producer].y ? add.x2 : add.x;
        reads.push_back(other);
        if (!disjoint(reads, add.y)) return;
        st.has_add = true;
        st.c = j;
        st.op = j;
        steps[j].kind = S_SKIP;
        st.name += "+add";
    };
    for (size_t i = 0; i < p.ops.size(); i++) {
        if (steps[i].kind == S_SKIP || steps[i].kind == S_GATE_UPADD) continue;
        const Op &op = p.ops[i];
        // depthwise -> pointwise
        if (op.kind == K_DWCONV && i + 1 < p.ops.size() && only_reader(u[i], i + 1)) {
            const Op &pw = p.ops[i + 1];
            if (pw.pointwise() && pw.x == op.y && pw.y != op.x) {
                DwPwArgs probe;
                probe.dw.c = int(op.oc);
                probe.oc = int(pw.oc);
                if (dw_pw_supported(probe)) {
                    Step &st = steps[i];
                    st.kind = S_DW_PW;
                    st.a = i;
                    st.b = i + 1;
                    st.op = i + 1;
                    st.name = "dw+pw";
                    steps[i + 1].kind = S_SKIP;
                    residual(st, i + 1, i + 1, {op.x});
                    continue;
                }
            }
        }
        // channelmul feeding a pointwise conv: the gate joins its input load
        if (op.kind == K_CHANNELMUL && i + 1 < p.ops.size() && only_reader(u[i], i + 1)) {
            const Op &pw = p.ops[i + 1];
            if (pw.pointwise() && pw.x == op.y && pw.n2 == 0 && disjoint({op.x, op.x2}, pw.y)) {
                Step &st = steps[i];
                st.kind = S_CONV;
                st.gated = true;
                st.a = i;
                st.b = i + 1;
                st.op = i + 1;
                st.srcs = {{op.x, op.ic, 0}};
                st.name = "gate+conv";
                steps[i + 1].kind = S_SKIP;
                residual(st, i + 1, i + 1, {op.x, op.x2});
                continue;
            }
        }
        // channelmul + add of its input: the RSE gate
        if (op.kind == K_CHANNELMUL && i + 1 < p.ops.size() && only_reader(u[i], i + 1)) {
            const Op &add = p.ops[i + 1];
            if (add.kind == K_ADD && ((add.x == op.y && add.x2 == op.x) || (add.x2 == op.y && add.x == op.x)) &&
                disjoint({op.x, op.x2}, add.y)) {
                Step &st = steps[i];
                st.kind = S_GATE_ADD;
                st.a = i;
                st.b = i + 1;
                st.op = i + 1;
                st.name = "gate_add";
                steps[i + 1].kind = S_SKIP;
                // an RSE output read only as the full-size input of an
                // upsample-add (the neck's top-down path): the gate-add runs
                // inside that upsample-add, at its place, from the conv
                // output and the gate, which must still hold their values
                const Uses &ua = u[i + 1];
                if (!ua.out && ua.readers.size() == 1) {
                    const size_t r = ua.readers[0];
                    const Op &up = p.ops[r];
                    if (up.kind == K_UPSAMPLEADD && up.x2 == add.y && up.x != add.y && intact(p, op.x, i + 1, r) &&
                        intact(p, op.x2, i + 1, r) && disjoint({up.x, op.x, op.x2}, up.y)) {
                        Step &su = steps[r];
                        su.kind = S_GATE_UPADD;
                        su.a = r;
                        su.b = i;
                        su.c = i + 1;
                        su.op = r;
                        su.name = "gate_add+upsample_add";
                        st.kind = S_SKIP;
                    }
                }
                continue;
            }
        }
        if (op.kind == K_CONV) {
            Step &st = steps[i];
            st.kind = S_CONV;
            st.b = i;
            std::vector<size_t> folded;
            std::vector<Step::Src> srcs;
            bool chained = false;
            if (!op.pointwise()) {
                chained = chain_sources(p, u, i, op.x, i, 0, srcs, folded);
                if (chained && op.n2 > 0) {
                    if (intact(p, op.x2, i, i)) srcs.push_back({op.x2, op.n2, 0});
                    chained = srcs.size() <= MAX_SOURCES;
                }
                if (chained && folded.empty()) chained = false;
                for (const Step::Src &src : srcs)
                    if (src.slot == op.y) chained = false;
            }
            if (chained) {
                st.srcs = srcs;
                for (size_t f : folded) steps[f].kind = S_SKIP;
                st.name = "conv(" + std::to_string(srcs.size()) + " sources)";
            } else {
                st.srcs = {{op.x, op.ic, 0}};
                if (op.n2) st.srcs.push_back({op.x2, op.n2, 0});
                st.name = "conv";
            }
            std::vector<size_t> reads;
            for (const Step::Src &src : st.srcs) reads.push_back(src.slot);
            residual(st, i, i, reads);
        }
    }
    return steps;
}

}  // namespace

namespace ppocr {
// The thread's last-error text, for entry points defined in other files.
void set_last_error(const std::string &msg) { g_error = msg; }
}  // namespace ppocr

// ------------------------------------------------------------------- model

// The lanes of one run, packed: every plan buffer holds the lanes' tensors
// back to back, pixel by pixel, sized for the largest total any operation
// writes there.
struct Group {
    std::vector<Plan> plans;            // one per distinct lane size
    std::vector<size_t> lane_plan;      // per lane: index into plans
    std::vector<size_t> in_off;         // per lane: first float of its input
    std::vector<std::vector<size_t>> out_off;  // per output, per lane: first float
    size_t in_floats = 0;
    std::vector<size_t> out_floats;     // per output: all lanes
    std::vector<std::unique_ptr<DeviceBuffer>> slots;
    DeviceBuffer mean_scratch, ctc_scratch, lane_tables;
    DeviceBuffer concat_scratch;  // a multi-source conv's input, written out for the tensor cores
    HostBuffer in_host;
    std::vector<std::unique_ptr<HostBuffer>> out_host;
    std::vector<std::function<int(cudaStream_t)>> launches;
    size_t input_slot = 0;
    std::vector<size_t> output_slots;
    float *slot_ptr(size_t s) const { return static_cast<float *>(slots[s]->p); }
    const Plan &lane(size_t n) const { return plans[lane_plan[n]]; }
    size_t count() const { return lane_plan.size(); }
};

struct ppocr_model {
    int device = 0;
    std::string name;
    bool integrated = false;
    cudaStream_t stream = nullptr;      // where the model runs
    cudaStream_t own_stream = nullptr;  // the stream it made
    cudaEvent_t done = nullptr;
    Plan plan;  // at the load size
    std::shared_ptr<Weights> weights;
    size_t weight_floats = 0;
    uint32_t options = 0;
    std::vector<Step> steps;
    bool steps_fused = false;
    std::vector<std::pair<size_t, size_t>> sizes;  // per lane (h, w)
    std::unique_ptr<Group> group;
    cudaGraphExec_t graph_host = nullptr, graph_device = nullptr;
    size_t launches = 0;
    bool pending = false;
    // Kernels record a nonzero code here when a bounded wait gives up
    // (page-locked and mapped, so reading it after a run costs no copy).
    int *err_host = nullptr, *err_dev = nullptr;

    ~ppocr_model() {
        if (device >= 0) cudaSetDevice(device);
        // Wait for this model's own work through its event: the stream may
        // belong to the caller (ppocr_model_set_stream) and be gone already.
        settle();
        if (own_stream) cudaStreamSynchronize(own_stream);
        drop_graphs();
        group.reset();
        if (done) cudaEventDestroy(done);
        if (own_stream) cudaStreamDestroy(own_stream);
        if (err_host) cudaFreeHost(err_host);
    }

    void settle() {
        if (pending && done) cudaEventSynchronize(done);
        pending = false;
    }

    void drop_graphs() {
        if (graph_host) cudaGraphExecDestroy(graph_host);
        if (graph_device) cudaGraphExecDestroy(graph_device);
        graph_host = graph_device = nullptr;
    }

    int bias_mode(const Op &op) const;
    int build_group(Group &g, std::string &err, Group *old);
    int record(bool copies);
    int enqueue(bool copies);
};

// Where the reference's tier-3 kernels add a convolution's bias: first for
// RGB stems (conv.rs:171-177), for pointwise layers with a multiple of 16
// output channels (pointwise.rs:77-102), for windowed ones of such width but
// the last `ow % 4` pixels of each row (dense.rs:60-66); last otherwise
// (pointwise.rs:33-35, dense.rs:127-130).
int ppocr_model::bias_mode(const Op &op) const {
    if (!op.pointwise() && op.ic == 3 && op.n2 == 0) return BIAS_FIRST;
    if (op.oc % 16) return BIAS_LAST;
    if (op.pointwise()) return BIAS_FIRST;
    return BIAS_FIRST_BUT_ROW_TAIL;
}

namespace {

// The lane table of operation `i` over the group's lanes, with the source
// shifts of a dense convolution's inputs (pixel prefix sums per source).
std::vector<LaneInfo> lane_table(const Group &g, size_t i, const std::vector<int> &shifts) {
    std::vector<LaneInfo> t(g.count());
    long pix = 0, ipix = 0, spix[MAX_SOURCES] = {0, 0, 0, 0}, tile = 0, run = 0, ftile = 0, row = 0;
    for (size_t n = 0; n < g.count(); n++) {
        const Op &op = g.lane(n).ops[i];
        LaneInfo &L = t[n];
        L.pix0 = pix;
        L.ipix0 = ipix;
        L.tile0 = tile;
        tile += (long(op.oh * op.ow) + 127) / 128;
        L.run0 = run;
        run += long(op.oh) * ((long(op.ow) + DW_RUN - 1) / DW_RUN);
        L.ftile0 = ftile;
        ftile += (long(op.oh * op.ow) + FOLD_OUT - 1) / FOLD_OUT;
        L.row0 = row;
        row += long(op.oh);
        for (int s = 0; s < MAX_SOURCES; s++) L.spix0[s] = spix[s];
        L.ih = int(op.ih); L.iw = int(op.iw); L.oh = int(op.oh); L.ow = int(op.ow);
        pix += long(op.oh * op.ow);
        ipix += long(op.ih * op.iw);
        for (size_t s = 0; s < shifts.size() && s < size_t(MAX_SOURCES); s++)
            spix[s] += long(op.ih >> shifts[s]) * long(op.iw >> shifts[s]);
    }
    return t;
}

// Row runs of DW_RUN output pixels over all lanes of a lane table.
long row_runs(const LaneInfo *t, int nl) {
    const LaneInfo &L = t[nl - 1];
    return L.run0 + long(L.oh) * ((long(L.ow) + DW_RUN - 1) / DW_RUN);
}

// A stride-1 conv whose output keeps its input's size (padding kh - 1 and
// kw - 1 in all): within a lane, each tap reads the input shifted by a
// constant number of packed pixels.
bool tc_windowed(const Op &op) {
    return op.kind == K_CONV && op.sh == 1 && op.sw == 1 && op.pt + op.pb == op.kh - 1 && op.pl + op.pr == op.kw - 1;
}

// A windowed 3-wide conv whose horizontal taps go into the tensor cores'
// columns (TcArgs::fold): whole 32-channel K blocks per vertical tap.
bool tc_foldable(const Op &op) {
    return tc_windowed(op) && op.kw == 3 && op.pl == 1 && (op.ic + op.n2) % 32 == 0 && op.oc <= 160;
}

long total_out(const Group &g, size_t i) {
    long m = 0;
    for (size_t n = 0; n < g.count(); n++) m += long(g.lane(n).ops[i].oh * g.lane(n).ops[i].ow);
    return m;
}

long total_in(const Group &g, size_t i) {
    long m = 0;
    for (size_t n = 0; n < g.count(); n++) m += long(g.lane(n).ops[i].ih * g.lane(n).ops[i].iw);
    return m;
}

}  // namespace

int ppocr_model::build_group(Group &g, std::string &err, Group *old) {
    const Plan &p0 = g.plans[0];
    const size_t N = g.count();
    int code = PPOCR_OK;
    g.input_slot = p0.slot;
    g.output_slots = p0.outputs;
    // Packed sizes: each buffer holds the most floats any writer puts there.
    std::vector<size_t> slot_floats(p0.pool.size(), 0);
    g.in_off.assign(N, 0);
    g.in_floats = 0;
    for (size_t n = 0; n < N; n++) {
        g.in_off[n] = g.in_floats;
        g.in_floats += g.lane(n).h * g.lane(n).w * g.lane(n).c;
    }
    slot_floats[p0.slot] = g.in_floats;
    for (size_t i = 0; i < p0.ops.size(); i++) {
        size_t total = 0;
        for (size_t n = 0; n < N; n++) total += g.lane(n).ops[i].out_len();
        slot_floats[p0.ops[i].y] = std::max(slot_floats[p0.ops[i].y], total);
    }
    g.out_off.assign(p0.outputs.size(), std::vector<size_t>(N, 0));
    g.out_floats.assign(p0.outputs.size(), 0);
    for (size_t k = 0; k < p0.outputs.size(); k++)
        for (size_t n = 0; n < N; n++) {
            g.out_off[k][n] = g.out_floats[k];
            g.out_floats[k] += g.lane(n).out_n[k];
        }
    // Tensors.
    g.slots.clear();
    for (size_t s = 0; s < slot_floats.size(); s++) {
        auto b = std::make_unique<DeviceBuffer>();
        DeviceBuffer *prev = old && s < old->slots.size() ? old->slots[s].get() : nullptr;
        if (!reserve(*b, prev, std::max<size_t>(slot_floats[s], 1) * sizeof(float), "allocating a tensor", code)) {
            err = g_error;
            return code;
        }
        g.slots.push_back(std::move(b));
    }
    // Scratch.
    const bool tc_allowed = !(options & PPOCR_OPT_NO_TENSOR_CORES);
    const int min_tiles = (options & PPOCR_OPT_THROUGHPUT) ? THROUGHPUT_TILES : 1;
    size_t mean_doubles = 1, ctc_floats = 1;
    for (size_t i = 0; i < p0.ops.size(); i++) {
        const Op &op = p0.ops[i];
        if (op.kind == K_MEAN) {
            long hw = 0;
            for (size_t n = 0; n < N; n++) hw = std::max<long>(hw, long(g.lane(n).ops[i].ih * g.lane(n).ops[i].iw));
            mean_doubles = std::max(mean_doubles, N * size_t(mean_chunks(hw, int(op.ic))) * op.ic);
        }
        if (op.kind == K_CTCHEAD || op.kind == K_CTCARGMAX) {
            size_t vocab = op.kind == K_CTCHEAD ? op.oc : op.n2;
            size_t cols = (vocab + 15) / 16 * 16;
            ctc_floats = std::max(ctc_floats, size_t(total_in(g, i)) * ctc_col_blocks(int(cols)) * 3);
            if (op.kind == K_CTCARGMAX && tc_allowed)
                ctc_floats = std::max(ctc_floats,
                                      size_t(total_in(g, i)) * 2 * tc_pointwise_slices(int(op.ic), int(cols)) * 3);
        }
    }
    // A windowed conv of several sources (or upsampled ones) on the tensor
    // cores reads them written out side by side.
    size_t concat_floats = 0;
    if (tc_allowed)
        for (const Step &st : steps) {
            if (st.kind == S_SKIP) continue;
            const size_t i = st.kind == S_CONV ? st.b : st.a;
            const Op &op = p0.ops[i];
            bool multi = op.kind == K_CONV && op.n2 > 0;
            if (st.kind == S_CONV) multi = st.srcs.size() > 1 || (!st.srcs.empty() && st.srcs[0].shift);
            if (multi && tc_windowed(op) && weights->tc_hi(i))
                concat_floats = std::max(concat_floats, size_t(total_in(g, i)) * (op.ic + op.n2));
        }
    if (concat_floats) {
        if (!reserve(g.concat_scratch, old ? &old->concat_scratch : nullptr, concat_floats * sizeof(float),
                     "allocating scratch", code)) {
            err = g_error;
            return code;
        }
    }
    if (!reserve(g.mean_scratch, old ? &old->mean_scratch : nullptr, mean_doubles * sizeof(double),
                 "allocating scratch", code) ||
        !reserve(g.ctc_scratch, old ? &old->ctc_scratch : nullptr, ctc_floats * sizeof(float), "allocating scratch",
                 code)) {
        err = g_error;
        return code;
    }
    // Page-locked host staging.
    if (!reserve(g.in_host, old ? &old->in_host : nullptr, std::max<size_t>(g.in_floats, 1) * sizeof(float),
                 "allocating host input", code)) {
        err = g_error;
        return code;
    }
    // Not cleared: the caller writes every lane's input before a run (a
    // reader writing the lanes on the GPU never touches this staging), and a
    // buffer kept from earlier sizes keeps its old contents, as the
    // reference's lanes do.
    g.out_host.clear();
    for (size_t k = 0; k < p0.outputs.size(); k++) {
        auto hb = std::make_unique<HostBuffer>();
        HostBuffer *prev = old && k < old->out_host.size() ? old->out_host[k].get() : nullptr;
        if (!reserve(*hb, prev, std::max<size_t>(g.out_floats[k], 1) * sizeof(float), "allocating host output",
                     code)) {
            err = g_error;
            return code;
        }
        // outputs are written by every run before they are read
        g.out_host.push_back(std::move(hb));
    }

    // Lane tables of every step, in one device array.
    std::vector<LaneInfo> tables;
    std::vector<size_t> table_at(steps.size(), 0);
    for (size_t k = 0; k < steps.size(); k++) {
        const Step &st = steps[k];
        if (st.kind == S_SKIP) continue;
        size_t i = st.kind == S_CONV ? st.b : st.a;
        std::vector<int> shifts;
        if (st.kind == S_CONV)
            for (const Step::Src &src : st.srcs) shifts.push_back(src.shift);
        else if (p0.ops[i].kind == K_CONV && p0.ops[i].n2)
            shifts = {0, 0};
        table_at[k] = tables.size();
        auto t = lane_table(g, i, shifts);
        tables.insert(tables.end(), t.begin(), t.end());
    }
    if (!reserve(g.lane_tables, old ? &old->lane_tables : nullptr, std::max<size_t>(tables.size(), 1) * sizeof(LaneInfo),
                 "allocating lane tables", code) ||
        // On the model's own stream, so that its kernels read the new tables:
        // a plain cudaMemcpy from pageable memory can return before its DMA
        // lands and is not ordered with a non-blocking stream, and a reused
        // buffer still holds the previous sizes' tables. The host vector is
        // staged before the call returns.
        !cuda_ok(cudaMemcpyAsync(g.lane_tables.p, tables.data(), tables.size() * sizeof(LaneInfo),
                                 cudaMemcpyHostToDevice, stream), "uploading lane tables", &code)) {
        err = g_error;
        return code;
    }
    const LaneInfo *lt = static_cast<const LaneInfo *>(g.lane_tables.p);

    // Launches.
    g.launches.clear();
    const Weights &W = *weights;
    const int nl = int(N);
    auto buf = [&g](size_t s) { return g.slot_ptr(s); };
    int *errp = err_dev;
    // A pointwise conv as the tensor-core kernel's arguments, when it goes
    // there. The choice depends on the layer alone, never on how many
    // pixels the run holds, so a lane gives the same bits alone as
    // alongside others.
    // Layers over per-lane vectors: a channel mean's output and the
    // pointwise convs that follow it (a squeeze-and-excite branch, one pixel
    // per lane at every size). They take the one-thread-per-output kernel;
    // a tensor-core launch there would be all set-up.
    std::vector<char> reads_vector(p0.ops.size(), 0);
    {
        std::vector<int> writer(p0.pool.size(), -1);
        std::vector<char> vector_out(p0.ops.size(), 0);
        for (size_t i = 0; i < p0.ops.size(); i++) {
            const Op &op = p0.ops[i];
            const int w = writer[op.x];
            reads_vector[i] = w >= 0 && vector_out[size_t(w)];
            vector_out[i] = op.kind == K_MEAN || (op.pointwise() && reads_vector[i]);
            writer[op.y] = int(i);
        }
    }
    // 0: not on the tensor cores; 1: there; 2: there, after the sources are
    // written out side by side (`gather`).
    auto tc_route = [&](size_t i, const ConvArgs &c, const LaneInfo *Lh, TcArgs &t, GatherArgs &gather) {
        if (!tc_allowed || !W.tc_hi(i)) return 0;
        const Op &op = p0.ops[i];
        const bool one = c.nsrc == 1 && !c.src[0].shift;
        const bool pw = one && c.kh == 1 && c.kw == 1 && c.sh == 1 && c.sw == 1 && !c.pt && !c.pl;
        if (!pw && (c.gate || !tc_windowed(op) || c.C % 32)) return 0;
        t.windowed = !pw;
        t.x = c.src[0].p;
        if (!pw && !one) {
            gather = GatherArgs();
            for (int q = 0; q < c.nsrc; q++) {
                gather.src[q] = c.src[q];
                if (c.src[q].c % 4) return 0;
            }
            gather.nsrc = c.nsrc; gather.C = c.C; gather.lanes = c.lanes; gather.nl = c.nl;
            gather.M = c.M;  // the output keeps the input's size
            gather.y = static_cast<float *>(g.concat_scratch.p);
            if (!gather.y || size_t(c.M) * c.C > concat_floats) return 0;
            t.x = gather.y;
        }
        t.C = c.C;
        t.kh = c.kh; t.kw = c.kw; t.pt = c.pt; t.pl = c.pl;
        t.lanes = c.lanes; t.nl = c.nl; t.gate = c.gate;
        const LaneInfo &last = Lh[c.nl - 1];
        t.tiles = last.tile0 + (long(last.oh) * last.ow + 127) / 128;
        t.w_hi = W.tc_hi(i); t.w_lo = W.tc_lo(i); t.b = c.b; t.res = c.res; t.y = c.y;
        t.M = c.M; t.K = c.kh * c.kw * c.C; t.N = c.oc; t.kpad = W.tc_kpad[i];
        if (W.tc_fold[i]) {
            if (pw) return 0;
            t.fold = true;
            t.tiles = last.ftile0 + (long(last.oh) * last.ow + FOLD_OUT - 1) / FOLD_OUT;
            t.K = c.kh * c.C;
            t.N = (c.oc + 15) / 16 * 48;
            t.toc = c.oc;
        }
        t.act = c.act; t.act2 = c.act2; t.err = errp;
        t.min_tiles = min_tiles;
        if (!tc_prepare(t)) return 0;
        return (!pw && !one) ? 2 : 1;
    };
    // Pushes a dense conv's launch: the tensor cores where the layer goes
    // there, else the FP32 implicit GEMM; `pre` runs first (a depthwise
    // layer whose output it reads, or nothing).
    auto push_conv = [&](size_t i, const ConvArgs &c0, const LaneInfo *Lh, std::function<int(cudaStream_t)> pre) {
        const Op &op = p0.ops[i];
        ConvArgs c = c0;
        c.out_rows = Lh[c.nl - 1].row0 + Lh[c.nl - 1].oh;
        for (int n = 0; n < c.nl; n++) c.max_ow = std::max(c.max_ow, Lh[n].ow);
        if (reads_vector[i] && op.pointwise() && c.nsrc == 1 && !c.src[0].shift) {
            // the same bits either way
            if (conv_vector_supported(c))
                g.launches.push_back([pre, c](cudaStream_t s) { return (pre ? pre(s) : 0) + launch_conv_vector(c, s); });
            else
                g.launches.push_back([pre, c](cudaStream_t s) { return (pre ? pre(s) : 0) + launch_conv(c, s); });
            return;
        }
        TcArgs t;
        GatherArgs ga;
        const int route = tc_route(i, c, Lh, t, ga);
        if (route == 2)
            g.launches.push_back([pre, ga, t](cudaStream_t s) {
                return (pre ? pre(s) : 0) + launch_gather(ga, s) + launch_tc(t, s);
            });
        else if (route == 1)
            g.launches.push_back([pre, t](cudaStream_t s) { return (pre ? pre(s) : 0) + launch_tc(t, s); });
        else
            g.launches.push_back([pre, c](cudaStream_t s) { return (pre ? pre(s) : 0) + launch_conv(c, s); });
    };
    for (size_t k = 0; k < steps.size(); k++) {
        const Step &st = steps[k];
        if (st.kind == S_SKIP) continue;
        const LaneInfo *L = lt + table_at[k];
        const LaneInfo *Lh = tables.data() + table_at[k];  // the same table on the host
        if (st.kind == S_DW_PW) {
            const Op &dw = p0.ops[st.a], &pw = p0.ops[st.b];
            DwPwArgs a;
            a.dw.x = buf(dw.x); a.dw.w = W.w(st.a); a.dw.b = W.b(st.a);
            a.dw.lanes = L; a.dw.nl = nl; a.dw.M = total_out(g, st.a); a.dw.c = int(dw.ic);
            a.dw.kh = int(dw.kh); a.dw.kw = int(dw.kw); a.dw.sh = int(dw.sh); a.dw.sw = int(dw.sw);
            a.dw.pt = int(dw.pt); a.dw.pl = int(dw.pl); a.dw.act = dw.fused;
            a.w2 = W.w(st.b); a.b2 = W.b(st.b); a.oc = int(pw.oc); a.act2 = pw.fused;
            a.bias_mode2 = bias_mode(pw);
            a.y = buf(pw.y);
            if (st.has_add) {
                const Op &add = p0.ops[st.c];
                a.res = buf(add.x == pw.y ? add.x2 : add.x);
                a.act3 = add.fused;
                a.y = buf(add.y);
            }
            // Without the tensor cores, narrow layers (24 to 96 channels in,
            // 24 to 96 out: the high-resolution blocks of both networks) take
            // the fused row-tile kernel: the depthwise map stays in shared
            // memory, both layers keep the exact FP32 order, and it runs
            // 1.7-2.2x faster than the tiled fused kernel below. Beside the
            // tensor cores it is slower than the depthwise row runs followed
            // by the pointwise tensor-core kernel, which keep those layers.
            if (!tc_allowed && pw.oc <= 96) {
                long rows = 0;
                int max_ow = 0;
                for (int n = 0; n < nl; n++) {
                    rows = std::max(rows, Lh[n].row0 + Lh[n].oh);
                    max_ow = std::max(max_ow, Lh[n].ow);
                }
                a.rows = rows;
                a.segs = 1;
                if (dwpw_tile_supported(a)) {
                    const int tp = dwpw_tile_pixels(a);
                    a.segs = (max_ow + tp - 1) / tp;
                    const bool quick = tc_allowed;
                    g.launches.push_back([a, quick](cudaStream_t s) { return launch_dwpw_tile(a, quick, s); });
                    continue;
                }
            }
            // Otherwise, with the tensor cores the depthwise layer runs alone
            // and the pointwise one on the tensor cores; without them, large
            // maps take the fused FP32 kernel and small ones the two FP32
            // kernels (the same bits either way).
            const bool tc_pw = tc_allowed && W.tc_hi(st.b);
            if (!tc_pw && a.dw.M >= DW_PW_MIN_PIXELS) {
                g.launches.push_back([a](cudaStream_t s) { return launch_dw_pw(a, s); });
                continue;
            }
            DwArgs d = a.dw;
            d.y = buf(dw.y);
            d.runs = row_runs(Lh, nl);
            d.quick = tc_allowed;
            ConvArgs c;
            c.src[0] = {buf(dw.y), int(dw.oc), 0};
            c.nsrc = 1;
            c.C = int(dw.oc);
            c.w = a.w2; c.b = a.b2;
            c.lanes = L; c.nl = nl; c.M = a.dw.M; c.oc = a.oc;
            c.act = a.act2; c.bias_mode = a.bias_mode2;
            c.res = a.res; c.act2 = a.act3;
            c.y = a.y;
            push_conv(st.b, c, Lh, [d](cudaStream_t s) { return launch_dw(d, s); });
            continue;
        }
        if (st.kind == S_CONV) {
            const Op &op = p0.ops[st.b];
            ConvArgs a;
            a.nsrc = int(st.srcs.size());
            a.C = 0;
            for (size_t q = 0; q < st.srcs.size(); q++) {
                a.src[q].p = buf(st.srcs[q].slot);
                a.src[q].c = int(st.srcs[q].c);
                a.src[q].shift = st.srcs[q].shift;
                a.C += int(st.srcs[q].c);
            }
            if (st.gated) a.gate = buf(p0.ops[st.a].x2);
            a.w = W.w(st.b); a.b = W.b(st.b);
            a.lanes = L; a.nl = nl; a.M = total_out(g, st.b); a.oc = int(op.oc);
            a.kh = int(op.kh); a.kw = int(op.kw); a.sh = int(op.sh); a.sw = int(op.sw);
            a.pt = int(op.pt); a.pl = int(op.pl);
            a.act = op.fused;
            a.bias_mode = bias_mode(op);
            a.quick = tc_allowed;  // stems: the quick quotient beside the tensor cores
            a.y = buf(op.y);
            if (st.has_add) {
                const Op &add = p0.ops[st.c];
                a.res = buf(add.x == op.y ? add.x2 : add.x);
                a.act2 = add.fused;
                a.y = buf(add.y);
            }
            push_conv(st.b, a, Lh, nullptr);
            continue;
        }
        if (st.kind == S_GATE_UPADD) {
            const Op &up = p0.ops[st.a], &cm = p0.ops[st.b], &add = p0.ops[st.c];
            EltArgs a;
            a.mode = ELT_GATE_UPSAMPLE_ADD;
            a.x = buf(up.x); a.x2 = buf(cm.x); a.g = buf(cm.x2); a.y = buf(up.y);
            a.lanes = L; a.nl = nl; a.M = total_out(g, st.a); a.c = int(up.oc); a.act = add.fused;
            a.sh = int(std::max<size_t>(up.sh, 1)); a.sw = int(std::max<size_t>(up.sw, 1));
            g.launches.push_back([a](cudaStream_t s) { return launch_elt(a, s); });
            continue;
        }
        if (st.kind == S_GATE_ADD) {
            const Op &cm = p0.ops[st.a], &add = p0.ops[st.b];
            EltArgs a;
            a.mode = ELT_GATE_ADD;
            a.x = buf(cm.x); a.x2 = buf(cm.x2); a.y = buf(add.y);
            a.lanes = L; a.nl = nl; a.M = total_out(g, st.a); a.c = int(cm.oc); a.act = add.fused;
            g.launches.push_back([a](cudaStream_t s) { return launch_elt(a, s); });
            continue;
        }
        // One operation alone.
        const size_t i = st.a;
        const Op &op = p0.ops[i];
        switch (op.kind) {
        case K_CONV: {
            ConvArgs a;
            a.src[0] = {buf(op.x), int(op.ic), 0};
            a.nsrc = 1;
            if (op.n2) { a.src[1] = {buf(op.x2), int(op.n2), 0}; a.nsrc = 2; }
            a.C = int(op.ic + op.n2);
            a.w = W.w(i); a.b = W.b(i);
            a.lanes = L; a.nl = nl; a.M = total_out(g, i); a.oc = int(op.oc);
            a.kh = int(op.kh); a.kw = int(op.kw); a.sh = int(op.sh); a.sw = int(op.sw);
            a.pt = int(op.pt); a.pl = int(op.pl); a.act = op.fused; a.bias_mode = bias_mode(op);
            a.quick = tc_allowed;
            a.y = buf(op.y);
            push_conv(i, a, Lh, nullptr);
            break;
        }
        case K_DWCONV: {
            DwArgs a;
            a.x = buf(op.x); a.w = W.w(i); a.b = W.b(i); a.y = buf(op.y);
            a.lanes = L; a.nl = nl; a.M = total_out(g, i); a.c = int(op.ic);
            a.kh = int(op.kh); a.kw = int(op.kw); a.sh = int(op.sh); a.sw = int(op.sw);
            a.pt = int(op.pt); a.pl = int(op.pl); a.act = op.fused;
            a.quick = tc_allowed;
            a.runs = row_runs(Lh, nl);
            g.launches.push_back([a](cudaStream_t s) { return launch_dw(a, s); });
            break;
        }
        case K_ADD: case K_CHANNELMUL: case K_CONCATC: case K_UPSAMPLE: case K_UPSAMPLEADD: {
            EltArgs a;
            a.mode = op.kind == K_ADD ? ELT_ADD : op.kind == K_CHANNELMUL ? ELT_CHANNELMUL
                     : op.kind == K_CONCATC ? ELT_CONCAT : op.kind == K_UPSAMPLE ? ELT_UPSAMPLE : ELT_UPSAMPLE_ADD;
            a.x = buf(op.x); a.x2 = op.has_second() ? buf(op.x2) : nullptr; a.y = buf(op.y);
            a.lanes = L; a.nl = nl; a.M = total_out(g, i);
            a.c = int(op.kind == K_CONCATC ? op.ic : op.oc); a.c2 = int(op.n2);
            a.sh = int(std::max<size_t>(op.sh, 1)); a.sw = int(std::max<size_t>(op.sw, 1)); a.act = op.fused;
            g.launches.push_back([a](cudaStream_t s) { return launch_elt(a, s); });
            break;
        }
        case K_MAXPOOL: case K_AVGPOOL: {
            PoolArgs a;
            a.x = buf(op.x); a.y = buf(op.y);
            a.lanes = L; a.nl = nl; a.M = total_out(g, i); a.c = int(op.ic);
            a.kh = int(op.kh); a.kw = int(op.kw); a.sh = int(op.sh); a.sw = int(op.sw);
            a.average = op.kind == K_AVGPOOL;
            g.launches.push_back([a](cudaStream_t s) { return launch_pool(a, s); });
            break;
        }
        case K_MEAN: {
            MeanArgs a;
            a.x = buf(op.x); a.y = buf(op.y); a.partial = static_cast<double *>(g.mean_scratch.p);
            a.lanes = L; a.nl = nl; a.c = int(op.ic);
            long hw = 0;
            for (size_t n = 0; n < N; n++) hw = std::max<long>(hw, long(g.lane(n).ops[i].ih * g.lane(n).ops[i].iw));
            a.chunks = mean_chunks(hw, a.c);
            g.launches.push_back([a](cudaStream_t s) { return launch_mean(a, s); });
            break;
        }
        case K_LAYERNORM: {
            LayerNormArgs a;
            a.x = buf(op.x); a.w = W.w(i); a.y = buf(op.y);
            a.pixels = int(total_out(g, i)); a.c = int(op.oc);
            a.fast = tc_allowed;
            g.launches.push_back([a](cudaStream_t s) { return launch_layernorm(a, s); });
            break;
        }
        case K_ATTENTION: {
            int tmax = 0;
            for (size_t n = 0; n < N; n++) tmax = std::max(tmax, int(g.lane(n).ops[i].iw));
            if (!attention_supported(tmax, int(op.oc), int(op.n2))) {
                err = "attention over " + std::to_string(tmax) + " steps with head size " +
                      std::to_string(op.oc / op.n2) + " exceeds this backend";
                return PPOCR_E_UNSUPPORTED;
            }
            AttentionArgs a;
            a.x = buf(op.x); a.y = buf(op.y); a.scale = W.w(i);
            a.lanes = L; a.nl = nl; a.tmax = tmax; a.c = int(op.oc); a.heads = int(op.n2);
            a.fast = tc_allowed;
            g.launches.push_back([a](cudaStream_t s) { return launch_attention(a, s); });
            break;
        }
        case K_CTCHEAD: case K_CTCARGMAX: {
            if (!ctc_supported(int(op.ic))) {
                err = "a CTC head over " + std::to_string(op.ic) + " input channels exceeds this backend";
                return PPOCR_E_UNSUPPORTED;
            }
            CtcArgs a;
            a.x = buf(op.x); a.w = W.w(i); a.b = W.b(i); a.y = buf(op.y);
            a.partial = static_cast<float *>(g.ctc_scratch.p);
            a.pixels = int(total_in(g, i)); a.ci = int(op.ic);
            a.probs = op.kind == K_CTCHEAD;
            a.vocab = int(a.probs ? op.oc : op.n2);
            a.cols = (a.vocab + 15) / 16 * 16;
            a.col_blocks = ctc_col_blocks(a.cols);
            if (!a.probs && tc_allowed && W.tc_hi(i)) {
                // the logits on the tensor cores, the classes checked exactly;
                // each CTA keeps its slice of the head's weights resident and
                // walks the time steps (streamed when that takes fewer slices)
                TcArgs t;
                t.x = a.x; t.C = t.K = a.ci; t.N = a.cols; t.kpad = W.tc_kpad[i];
                t.w_hi = W.tc_hi(i); t.w_lo = W.tc_lo(i); t.b = a.b; t.y = a.y;
                t.M = a.pixels; t.lanes = L; t.nl = nl; t.err = errp;
                t.vocab = a.vocab; t.partial = a.partial;
                CtcMergeArgs mg;
                mg.partial = a.partial; mg.x = a.x; mg.w = a.w; mg.b = a.b; mg.y = a.y;
                mg.pixels = a.pixels; mg.ci = a.ci; mg.vocab = a.vocab;
                mg.wmax = W.tc_wmax[i]; mg.bmax = W.tc_bmax[i];
                t.min_tiles = min_tiles;
                // the path depends on the layer's own need, never on how
                // large a reused scratch buffer happens to be
                if (tc_prepare(t) && size_t(a.pixels) * t.blocks * 3 <= ctc_floats) {
                    mg.blocks = t.blocks; mg.bn = t.bn;
                    g.launches.push_back(
                        [t, mg](cudaStream_t s) { return launch_tc(t, s) + launch_ctc_tc_merge(mg, s); });
                    break;
                }
            }
            g.launches.push_back([a](cudaStream_t s) { return launch_ctc(a, s); });
            break;
        }
        case K_CONVTRANSPOSE: {
            ConvTArgs a;
            a.x = buf(op.x); a.w = W.w(i); a.b = W.b(i); a.y = buf(op.y);
            a.lanes = L; a.nl = nl; a.Min = total_in(g, i); a.ic = int(op.ic); a.oc = int(op.oc);
            a.kh = int(op.kh); a.kw = int(op.kw); a.act = op.fused;
            a.bias_first = (op.kh * op.kw * op.oc) % 16 == 0;
            if (tc_allowed && W.tc_hi(i)) {
                // a pointwise GEMM ic -> kh*kw*oc whose epilogue places each
                // column in its output pixel
                TcArgs t;
                t.x = a.x; t.C = t.K = a.ic; t.N = a.kh * a.kw * a.oc; t.kpad = W.tc_kpad[i];
                t.w_hi = W.tc_hi(i); t.w_lo = W.tc_lo(i); t.b = a.b; t.y = a.y;
                t.M = a.Min; t.lanes = L; t.nl = nl; t.act = a.act; t.err = errp;
                t.tkh = a.kh; t.tkw = a.kw; t.toc = a.oc;
                t.min_tiles = min_tiles;
                if (tc_prepare(t)) {
                    g.launches.push_back([t](cudaStream_t s) { return launch_tc(t, s); });
                    break;
                }
            }
            g.launches.push_back([a](cudaStream_t s) { return launch_convt(a, s); });
            break;
        }
        default:
            err = std::string("operation kind ") + kind_name(op.kind) + " is not supported";
            return PPOCR_E_UNSUPPORTED;
        }
    }
    return PPOCR_OK;
}

// Record one run on the stream: the input copies (when `copies`), every
// step's kernels, the output copies.
int ppocr_model::record(bool copies) {
    Group &g = *group;
    if (copies) {
        if (!cuda_ok(cudaMemcpyAsync(g.slot_ptr(g.input_slot), g.in_host.p, g.in_floats * sizeof(float),
                                     cudaMemcpyHostToDevice, stream), "copying the input"))
            return PPOCR_E_DEVICE;
    }
    size_t count = 0;
    for (auto &l : g.launches) count += size_t(l(stream));
    if (copies) {
        for (size_t k = 0; k < g.output_slots.size(); k++) {
            if (!cuda_ok(cudaMemcpyAsync(g.out_host[k]->p, g.slot_ptr(g.output_slots[k]),
                                         g.out_floats[k] * sizeof(float), cudaMemcpyDeviceToHost, stream),
                         "copying an output"))
                return PPOCR_E_DEVICE;
        }
    }
    launches = count;
    if (!cuda_ok(cudaGetLastError(), "launching a kernel")) return PPOCR_E_DEVICE;
    return PPOCR_OK;
}

int ppocr_model::enqueue(bool copies) {
    if (!cuda_ok(cudaSetDevice(device), "selecting the device")) return PPOCR_E_DEVICE;
    if (!group) return fail(PPOCR_E_SIZE, "the model has no lanes");
    if (pending) settle();  // the error word belongs to one run at a time
    if (err_host) *reinterpret_cast<volatile int *>(err_host) = 0;
    int rc;
    if (options & PPOCR_OPT_NO_GRAPH) {
        rc = record(copies);
        if (rc) return rc;
    } else {
        cudaGraphExec_t &exec = copies ? graph_host : graph_device;
        if (!exec) {
            cudaGraph_t graph = nullptr;
            if (!cuda_ok(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "capturing the run"))
                return PPOCR_E_DEVICE;
            rc = record(copies);
            cudaError_t e = cudaStreamEndCapture(stream, &graph);
            if (rc) {
                if (graph) cudaGraphDestroy(graph);
                return rc;
            }
            if (!cuda_ok(e, "capturing the run")) return PPOCR_E_DEVICE;
            e = cudaGraphInstantiate(&exec, graph, 0);
            cudaGraphDestroy(graph);
            if (!cuda_ok(e, "instantiating the run")) return PPOCR_E_DEVICE;
        }
        if (!cuda_ok(cudaGraphLaunch(exec, stream), "launching the run")) return PPOCR_E_DEVICE;
    }
    if (!cuda_ok(cudaEventRecord(done, stream), "recording completion")) return PPOCR_E_DEVICE;
    pending = true;
    return PPOCR_OK;
}

// ------------------------------------------------------------------- C ABI

namespace {

int make_model(Plan &&plan, std::shared_ptr<Weights> weights, size_t weight_floats, int device, ppocr_model **out) {
    auto m = std::make_unique<ppocr_model>();
    m->device = device;
    m->plan = std::move(plan);
    m->weights = std::move(weights);
    m->weight_floats = weight_floats;
    cudaDeviceProp prop;
    if (!cuda_ok(cudaSetDevice(device), "selecting the device") ||
        !cuda_ok(cudaGetDeviceProperties(&prop, device), "reading the device"))
        return PPOCR_E_DEVICE;
    m->name = prop.name;
    m->integrated = prop.integrated != 0;
    configure_device(device);
    if (!cuda_ok(cudaStreamCreateWithFlags(&m->own_stream, cudaStreamNonBlocking), "creating a stream") ||
        !cuda_ok(cudaEventCreateWithFlags(&m->done, cudaEventDisableTiming), "creating an event") ||
        !cuda_ok(cudaHostAlloc(reinterpret_cast<void **>(&m->err_host), sizeof(int), cudaHostAllocMapped),
                 "allocating the error word") ||
        !cuda_ok(cudaHostGetDevicePointer(reinterpret_cast<void **>(&m->err_dev), m->err_host, 0),
                 "mapping the error word"))
        return PPOCR_E_DEVICE;
    *m->err_host = 0;
    m->stream = m->own_stream;
    uint32_t hw[2] = {uint32_t(m->plan.h), uint32_t(m->plan.w)};
    int rc = ppocr_model_set_sizes(m.get(), hw, 1);
    if (rc) return rc;
    *out = m.release();
    return PPOCR_OK;
}

}  // namespace

extern "C" {

int ppocr_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

const char *ppocr_last_error(void) { return g_error.c_str(); }

int ppocr_model_load_bytes(const void *bytes, size_t len, int device, ppocr_model **out) {
    g_error.clear();
    if (!bytes || !out) return fail(PPOCR_E_ARG, "null argument");
    *out = nullptr;
    // The plan is checked before any device is touched.
    Plan plan;
    std::vector<float> values;
    std::string err;
    if (!Plan::parse(static_cast<const uint8_t *>(bytes), len, plan, values, err)) return fail(PPOCR_E_PLAN, err);
    int count = ppocr_device_count();
    if (device < 0 || device >= count)
        return fail(PPOCR_E_DEVICE, "device " + std::to_string(device) + " of " + std::to_string(count));
    if (!cuda_ok(cudaSetDevice(device), "selecting the device")) return PPOCR_E_DEVICE;
    // Re-pack every block on a 256-byte boundary.
    auto w = std::make_shared<Weights>();
    w->device = device;
    std::vector<float> arena;
    auto place = [&](size_t at, size_t n) {
        if (!n) return SIZE_MAX;
        while (arena.size() % 64) arena.push_back(0.0f);
        size_t where = arena.size();
        arena.insert(arena.end(), values.begin() + at, values.begin() + at + n);
        return where;
    };
    for (const Op &op : plan.ops) {
        w->w_at.push_back(place(op.w0, op.w1));
        w->b_at.push_back(place(op.b0, op.b1));
    }
    arena.resize(std::max<size_t>(arena.size(), 1) + 64, 0.0f);
    // Tensor-core copies of the dense convolutions' weights, W [k][n] (k over
    // kh, kw, C), and of the CTC argmax heads', W [n/16][k][16]: to
    // [n][kpad], the high tf32 half (low 13 mantissa bits cleared) and the
    // exact remainder.
    std::vector<float> tc;
    for (const Op &op : plan.ops) {
        size_t hi = SIZE_MAX, lo = SIZE_MAX;
        int kpad = 0;
        float wmax = 0.0f, bmax = 0.0f;
        const bool ctc = op.kind == K_CTCARGMAX && op.w1;
        const bool convt = op.kind == K_CONVTRANSPOSE && op.w1;  // [ic][kh][kw][oc]: K = ic
        const bool fold = op.w1 && tc_foldable(op);
        const int C = int(op.ic + op.n2);
        int K = ctc || convt ? int(op.ic) : int(op.kh * op.kw * C);
        int N = ctc ? int((op.n2 + 15) / 16 * 16) : convt ? int(op.kh * op.kw * op.oc) : int(op.oc);
        if (fold) {
            K = int(op.kh) * C;
            N = int((op.oc + 15) / 16) * 48;
        }
        if (((op.kind == K_CONV || convt) && op.w1 && tc_weights_wanted(K, N)) || ctc) {
            kpad = pw_tc_kpad(K);
            while (tc.size() % 64) tc.push_back(0.0f);
            hi = tc.size();
            lo = hi + size_t(N) * kpad;
            tc.resize(lo + size_t(N) * kpad, 0.0f);
            for (int n = 0; n < N; n++)
                for (int k = 0; k < K; k++) {
                    size_t at = ctc ? (size_t(n / 16) * K + k) * 16 + n % 16 : size_t(k) * N + n;
                    if (fold) {
                        // column 48 j + 16 kx + e: channel 16 j + e of tap (ky, kx), k = ky * C + c
                        const int o = n / 48 * 16 + n % 16, kx = n % 48 / 16, ky = k / C, c = k % C;
                        if (o >= int(op.oc)) continue;
                        at = (size_t(ky * 3 + kx) * C + c) * op.oc + o;
                    }
                    float v = values[op.w0 + at];
                    uint32_t u;
                    std::memcpy(&u, &v, 4);
                    u &= 0xFFFFE000u;
                    float h;
                    std::memcpy(&h, &u, 4);
                    tc[hi + size_t(n) * kpad + k] = h;
                    tc[lo + size_t(n) * kpad + k] = v - h;
                    if (ctc && n < int(op.n2)) wmax = std::max(wmax, std::fabs(v));
                }
            if (ctc)
                for (int n = 0; n < int(op.n2); n++) bmax = std::max(bmax, std::fabs(values[op.b0 + size_t(n)]));
        }
        w->tc_hi_at.push_back(hi);
        w->tc_lo_at.push_back(lo);
        w->tc_kpad.push_back(kpad);
        w->tc_wmax.push_back(wmax);
        w->tc_bmax.push_back(bmax);
        w->tc_fold.push_back(fold && hi != SIZE_MAX);
    }
    tc.resize(std::max<size_t>(tc.size(), 1) + 64, 0.0f);
    int code = PPOCR_E_DEVICE;
    w->arena.bytes = arena.size() * sizeof(float);
    if (!cuda_ok(cudaMalloc(&w->arena.p, w->arena.bytes), "allocating weights", &code)) return code;
    if (!cuda_ok(cudaMemcpy(w->arena.p, arena.data(), w->arena.bytes, cudaMemcpyHostToDevice), "uploading weights"))
        return PPOCR_E_DEVICE;
    w->tc_arena.bytes = tc.size() * sizeof(float);
    if (!cuda_ok(cudaMalloc(&w->tc_arena.p, w->tc_arena.bytes), "allocating weights", &code)) return code;
    if (!cuda_ok(cudaMemcpy(w->tc_arena.p, tc.data(), w->tc_arena.bytes, cudaMemcpyHostToDevice),
                 "uploading weights"))
        return PPOCR_E_DEVICE;
    // A copy from pageable memory may return before its DMA lands; the
    // weights are complete before any stream of any model reads them.
    if (!cuda_ok(cudaDeviceSynchronize(), "uploading weights")) return PPOCR_E_DEVICE;
    return make_model(std::move(plan), w, values.size(), device, out);
}

int ppocr_model_load(const char *plan_path, int device, ppocr_model **out) {
    g_error.clear();
    if (!plan_path || !out) return fail(PPOCR_E_ARG, "null argument");
    std::ifstream f(plan_path, std::ios::binary);
    if (!f) return fail(PPOCR_E_PLAN, std::string("reading the plan: cannot open ") + plan_path);
    std::vector<char> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    return ppocr_model_load_bytes(bytes.data(), bytes.size(), device, out);
}

int ppocr_model_share_weights(const ppocr_model *src, ppocr_model **out) {
    g_error.clear();
    if (!src || !out) return fail(PPOCR_E_ARG, "null argument");
    *out = nullptr;
    Plan plan = src->plan;
    std::string err;
    return make_model(std::move(plan), src->weights, src->weight_floats, src->device, out);
}

void ppocr_model_free(ppocr_model *model) { delete model; }

const char *ppocr_model_device_name(const ppocr_model *m) { return m ? m->name.c_str() : ""; }
int ppocr_model_integrated(const ppocr_model *m) { return m && m->integrated ? 1 : 0; }
size_t ppocr_model_max_lanes(const ppocr_model *m) { return m ? 256 : 0; }
size_t ppocr_model_output_count(const ppocr_model *m) { return m ? m->plan.outputs.size() : 0; }

int ppocr_model_set_input_size(ppocr_model *m, uint32_t height, uint32_t width) {
    uint32_t hw[2] = {height, width};
    return ppocr_model_set_sizes(m, hw, 1);
}

int ppocr_model_set_sizes(ppocr_model *m, const uint32_t *hw, size_t lanes) {
    g_error.clear();
    if (!m || (!hw && lanes)) return fail(PPOCR_E_ARG, "null argument");
    if (lanes == 0) return fail(PPOCR_E_SIZE, "no lanes");
    if (lanes > ppocr_model_max_lanes(m))
        return fail(PPOCR_E_SIZE, std::to_string(lanes) + " lanes, more than the " +
                                      std::to_string(ppocr_model_max_lanes(m)) + " a run takes");
    if (!cuda_ok(cudaSetDevice(m->device), "selecting the device")) return PPOCR_E_DEVICE;
    m->settle();
    // Every size is checked first, so that a refusal leaves the model as it was.
    std::map<std::pair<size_t, size_t>, size_t> plan_of;
    std::vector<std::pair<size_t, size_t>> sizes;
    auto g = std::make_unique<Group>();
    for (size_t l = 0; l < lanes; l++) {
        std::pair<size_t, size_t> s{hw[2 * l], hw[2 * l + 1]};
        auto it = plan_of.find(s);
        if (it == plan_of.end()) {
            Plan p = m->plan;
            std::string err;
            if (!p.set_size(s.first, s.second, m->weight_floats, err)) return fail(PPOCR_E_SIZE, err);
            it = plan_of.emplace(s, g->plans.size()).first;
            g->plans.push_back(std::move(p));
        }
        g->lane_plan.push_back(it->second);
        sizes.push_back(s);
    }
    bool fused = !(m->options & PPOCR_OPT_NO_FUSION);
    if (m->steps.empty() || m->steps_fused != fused) {
        m->steps = fuse(m->plan, fused);
        m->steps_fused = fused;
    }
    m->drop_graphs();
    std::string err;
    int rc = m->build_group(*g, err, m->group.get());
    if (rc) return fail(rc, err);
    m->group = std::move(g);
    m->sizes = std::move(sizes);
    return PPOCR_OK;
}

float *ppocr_model_lane_input(ppocr_model *m, size_t lane, size_t *len) {
    if (!m || !m->group || lane >= m->group->count()) {
        fail(PPOCR_E_ARG, "no such lane");
        return nullptr;
    }
    const Group &g = *m->group;
    const Plan &p = g.lane(lane);
    if (len) *len = p.h * p.w * p.c;
    return static_cast<float *>(g.in_host.p) + g.in_off[lane];
}

const float *ppocr_model_lane_output(const ppocr_model *m, size_t lane, size_t index, size_t *len) {
    if (!m || !m->group || lane >= m->group->count() || index >= m->plan.outputs.size()) {
        fail(PPOCR_E_ARG, "no such lane or output");
        return nullptr;
    }
    const Group &g = *m->group;
    if (len) *len = g.lane(lane).out_n[index];
    return static_cast<const float *>(g.out_host[index]->p) + g.out_off[index][lane];
}

float *ppocr_model_lane_device_input(ppocr_model *m, size_t lane, size_t *len) {
    if (!m || !m->group || lane >= m->group->count()) {
        fail(PPOCR_E_ARG, "no such lane");
        return nullptr;
    }
    const Group &g = *m->group;
    const Plan &p = g.lane(lane);
    if (len) *len = p.h * p.w * p.c;
    return g.slot_ptr(g.input_slot) + g.in_off[lane];
}

const float *ppocr_model_lane_device_output(const ppocr_model *m, size_t lane, size_t index, size_t *len) {
    if (!m || !m->group || lane >= m->group->count() || index >= m->plan.outputs.size()) {
        fail(PPOCR_E_ARG, "no such lane or output");
        return nullptr;
    }
    const Group &g = *m->group;
    if (len) *len = g.lane(lane).out_n[index];
    return g.slot_ptr(g.output_slots[index]) + g.out_off[index][lane];
}

int ppocr_model_enqueue(ppocr_model *m) {
    g_error.clear();
    if (!m) return fail(PPOCR_E_ARG, "null model");
    return m->enqueue(true);
}

int ppocr_model_enqueue_device(ppocr_model *m) {
    g_error.clear();
    if (!m) return fail(PPOCR_E_ARG, "null model");
    return m->enqueue(false);
}

// Poll the completion event until it fires or the deadline passes; the
// reference waits forever (vk.rs:373-378).
int ppocr_model_wait(ppocr_model *m, uint32_t timeout_ms) {
    g_error.clear();
    if (!m) return fail(PPOCR_E_ARG, "null model");
    if (!m->pending) return PPOCR_OK;
    auto start = std::chrono::steady_clock::now();
    for (unsigned spin = 0;; spin++) {
        cudaError_t e = cudaEventQuery(m->done);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady) {
            m->pending = false;
            return cuda_ok(e, "running the network") ? PPOCR_OK : PPOCR_E_DEVICE;
        }
        if (timeout_ms) {
            auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - start);
            if (ms.count() >= timeout_ms)
                return fail(PPOCR_E_TIMEOUT, "the GPU did not finish within " + std::to_string(timeout_ms) + " ms");
        }
        if (spin < 2000)
            std::this_thread::yield();
        else
            std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    m->pending = false;
    if (m->err_host && *reinterpret_cast<volatile int *>(m->err_host))
        return fail(PPOCR_E_DEVICE, "a tensor-core kernel gave up waiting for its MMAs (bounded wait expired)");
    return PPOCR_OK;
}

int ppocr_model_run(ppocr_model *m, uint32_t timeout_ms) {
    int rc = ppocr_model_enqueue(m);
    if (rc) return rc;
    return ppocr_model_wait(m, timeout_ms);
}

void *ppocr_model_stream(ppocr_model *m) { return m ? static_cast<void *>(m->stream) : nullptr; }

int ppocr_model_set_stream(ppocr_model *m, void *stream) {
    g_error.clear();
    if (!m) return fail(PPOCR_E_ARG, "null model");
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m->own_stream;
    if (s == m->stream) return PPOCR_OK;
    m->settle();
    // uploads queued on the old stream (the lane tables) land before the
    // new stream's kernels read them
    if (!cuda_ok(cudaSetDevice(m->device), "selecting the device") ||
        !cuda_ok(cudaStreamSynchronize(m->stream), "switching streams"))
        return PPOCR_E_DEVICE;
    m->stream = s;
    m->drop_graphs();
    return PPOCR_OK;
}

int ppocr_model_set_options(ppocr_model *m, uint32_t options) {
    g_error.clear();
    if (!m) return fail(PPOCR_E_ARG, "null model");
    if (options == m->options) return PPOCR_OK;
    bool refuse = (options ^ m->options) & (PPOCR_OPT_NO_FUSION | PPOCR_OPT_NO_TENSOR_CORES | PPOCR_OPT_THROUGHPUT);
    m->options = options;
    m->drop_graphs();
    if (refuse && !m->sizes.empty()) {
        std::vector<uint32_t> hw;
        for (auto &s : m->sizes) {
            hw.push_back(uint32_t(s.first));
            hw.push_back(uint32_t(s.second));
        }
        return ppocr_model_set_sizes(m, hw.data(), m->sizes.size());
    }
    return PPOCR_OK;
}

// Counted when the run is recorded (each launch function returns how many
// kernels it started); 0 before the first run at the current sizes.
size_t ppocr_model_launches(const ppocr_model *m) { return m ? m->launches : 0; }

const char *ppocr_model_step_name(const ppocr_model *m, size_t i) {
    if (!m) return nullptr;
    size_t k = 0;
    for (const Step &st : m->steps) {
        if (st.kind == S_SKIP) continue;
        if (k++ == i) return st.name.c_str();
    }
    return nullptr;
}

}  // extern "C"
