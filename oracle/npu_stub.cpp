// The reference's src/xdna-exec.cpp names the NPU service's methods, which
// live in src/xdna-npu.cpp together with the XRT driver plumbing. The
// oracle's reference build runs pieces with no NPU (a null xdna_npu, the
// reference's host path), so none of these is ever called; they exist so the
// build links. Each reports failure if it ever were. TEST INFRASTRUCTURE ONLY.
#include "xdna-npu.h"

#include <cstdio>
#include <cstdlib>

namespace {
[[noreturn]] void not_here(const char *what) {
    fprintf(stderr, "oracle reference build: xdna_npu::%s called, but this build has no NPU\n", what);
    abort();
}
}  // namespace

bool xdna_npu::wkey::operator<(const wkey &o) const {
    if (buffer != o.buffer) return buffer < o.buffer;
    if (data != o.data) return data < o.data;
    if (type != o.type) return type < o.type;
    if (K != o.K) return K < o.K;
    return N < o.N;
}
bool xdna_npu::has_fused_shape(int64_t, int64_t) { not_here("has_fused_shape"); }
bool xdna_npu::reserve(int, const std::vector<std::vector<wkey>> &, std::string &) { not_here("reserve"); }
bool xdna_npu::begin(int, const std::vector<wkey> &, int64_t, std::string &) { not_here("begin"); }
void xdna_npu::encode_row(int, int64_t, const float *) { not_here("encode_row"); }
bool xdna_npu::submit(int, std::string &) { not_here("submit"); }
bool xdna_npu::wait(int, std::string &) { not_here("wait"); }
bool xdna_npu::decode_row(int, int, int64_t, float *) const { not_here("decode_row"); }
const char *xdna_npu::not_finite_error() { return "oracle reference build: a non-finite result"; }
