// PPOCRPL1 plan: parsing, shape derivation and every consistency check the
// reference applies before running anything (ppocr-native
// `src/engine/plan.rs:296-842`). A plan is never trusted.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace ppocr {

enum Kind : int {
    K_CONV, K_DWCONV, K_ADD, K_MAXPOOL, K_AVGPOOL, K_CHANNELMUL, K_CONCATC,
    K_LAYERNORM, K_ATTENTION, K_MEAN, K_CTCHEAD, K_CTCARGMAX, K_UPSAMPLE,
    K_UPSAMPLEADD, K_CONVTRANSPOSE, K_COUNT
};

// Folded activations, plan.rs:149-175; A_HARDSWISH (7) is this library's
// extension, x * hardsigmoid(x).
enum Act : int {
    A_NONE, A_RELU, A_SIGMOID, A_GELU, A_SWISH, A_HARDSIGMOID, A_HARDSIGMOIDFIFTH,
    A_HARDSWISH, A_COUNT
};

const char *kind_name(int kind);

struct Op {
    int kind = 0, fused = 0;
    size_t x = 0, x2 = 0, y = 0;
    size_t ih = 0, iw = 0, ic = 0, oh = 0, ow = 0, oc = 0;
    size_t kh = 0, kw = 0, sh = 0, sw = 0;
    long pt = 0, pb = 0, pl = 0, pr = 0;
    size_t n2 = 0;
    size_t w0 = 0, w1 = 0, b0 = 0, b1 = 0;  // weight / bias blocks, in floats

    bool pointwise() const {
        return kind == K_CONV && kh == 1 && kw == 1 && sh == 1 && sw == 1 && !pt && !pb && !pl && !pr;
    }
    bool has_second() const {
        return kind == K_ADD || kind == K_CHANNELMUL || kind == K_CONCATC || kind == K_UPSAMPLEADD ||
               (kind == K_CONV && n2 > 0);
    }
    size_t out_len() const { return oh * ow * oc; }
    size_t in_len() const { return ih * iw * ic; }
};

struct Plan {
    size_t slot = 0, h = 0, w = 0, c = 0;  // input buffer and size
    std::vector<size_t> outputs;           // buffer of each output
    std::vector<size_t> out_n;             // elements of each output
    std::vector<size_t> pool;              // floats each buffer holds
    std::vector<Op> ops;

    // Parse and check; weights receive the decoded floats (subnormals
    // flushed to signed zero, non-finite values refused).
    static bool parse(const uint8_t *bytes, size_t len, Plan &plan, std::vector<float> &weights,
                      std::string &err);
    // Re-derive shapes for an input height x width and check; on failure
    // the plan keeps its size (plan.rs:383-398).
    bool set_size(size_t height, size_t width, size_t weight_floats, std::string &err);

  private:
    bool derive_shapes(size_t height, size_t width, std::string &err);
    bool check(size_t weight_floats, std::string &err) const;
    bool produced(size_t before, size_t slot, size_t &h, size_t &w, size_t &c) const;
};

}  // namespace ppocr
