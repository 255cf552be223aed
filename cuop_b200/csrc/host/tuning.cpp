// GEMM variant selection table (the replacement of the reference's size
// thresholds, src/cuda_op/detail/cuBlas/gemm.cu:305-356, and of its
// AutoTuner-driven kernel choice, src/jit/Blas/gemm_jit_plugin.cu:667-738).
//
// A table is plain text, one rule per line, '#' starts a comment:
//
//   dtype  transA  transB  M      N      K      batch  variant
//   bf16   0       0       256:   256:   256:   1:1    tc2
//   f32    *       *       *      :255   *      *      ffma
//
// dtype is f32, f64, f16, bf16 or *; transA / transB are 0, 1 or *; each
// size field is `lo:hi` (inclusive; an empty side is unbounded) or `*`;
// variant is one of the names of gemm_variant_name().  The first matching
// row wins; a variant that cannot run the problem (alignment, dtype) falls
// back to the built-in choice.  Tables are produced by the offline sweep
// (cuop_b200/tuning.py) and loaded at start-up by the hosts.
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <memory>
#include <mutex>
#include <sstream>
#include <string>
#include <vector>

#include "cuopx.h"
#include "dispatch.h"

namespace cuopx {

namespace {

const char* const kVariantNames[kVariantCount] = {"auto",          "tc2",           "tc_128x256",
                                                  "tc_128x128",    "tf32x3_128x64", "tf32x3_128x128",
                                                  "ffma",          "generic",       "tc2_256x512",
                                                  "tc_128x128_2cta", "tc_128x64_2cta", "tf32x3_128x128_k2",
                                                  "tc2_256x128",   "tf32x3_256x128_pair"};

struct Range {
  int64_t lo = 0, hi = INT64_MAX;
  bool has(int64_t v) const { return v >= lo && v <= hi; }
};

struct Rule {
  int dtype = -1;  // -1: any
  int transA = -1, transB = -1;
  Range m, n, k, batch;
  int variant = kVariantAuto;
};

using Table = std::vector<Rule>;

std::mutex g_table_mu;
std::shared_ptr<const Table> g_table;  // replaced whole; readers take a copy of the pointer
std::atomic<int> g_forced{kVariantAuto};
thread_local int t_hint = kVariantAuto;  // per-thread override (plugins' kernel_type)

bool parse_range(const std::string& tok, Range& r) {
  if (tok == "*") return true;
  const auto colon = tok.find(':');
  if (colon == std::string::npos) return false;
  const std::string lo = tok.substr(0, colon), hi = tok.substr(colon + 1);
  char* end = nullptr;
  if (!lo.empty()) {
    r.lo = std::strtoll(lo.c_str(), &end, 10);
    if (*end) return false;
  }
  if (!hi.empty()) {
    r.hi = std::strtoll(hi.c_str(), &end, 10);
    if (*end) return false;
  }
  return r.lo <= r.hi;
}

bool parse_flag(const std::string& tok, int& out) {
  if (tok == "*") return (out = -1), true;
  if (tok == "0" || tok == "1") return (out = tok[0] - '0'), true;
  return false;
}

int variant_by_name(const char* name) {
  for (int v = 0; v < kVariantCount; ++v)
    if (std::strcmp(name, kVariantNames[v]) == 0) return v;
  return -1;
}

// Returns 0 and fills `t`, or the 1-based number of the first bad line.
int parse_table(const char* text, Table& t) {
  std::istringstream in(text);
  std::string line;
  int lineno = 0;
  while (std::getline(in, line)) {
    ++lineno;
    const auto hash = line.find('#');
    if (hash != std::string::npos) line.resize(hash);
    std::istringstream ls(line);
    std::vector<std::string> tok;
    for (std::string w; ls >> w;) tok.push_back(w);
    if (tok.empty()) continue;
    if (tok.size() != 8) return lineno;
    Rule r;
    if (tok[0] == "*") r.dtype = -1;
    else if (tok[0] == "f32") r.dtype = CUOPX_F32;
    else if (tok[0] == "f64") r.dtype = CUOPX_F64;
    else if (tok[0] == "f16") r.dtype = CUOPX_F16;
    else if (tok[0] == "bf16") r.dtype = CUOPX_BF16;
    else return lineno;
    if (!parse_flag(tok[1], r.transA) || !parse_flag(tok[2], r.transB)) return lineno;
    if (!parse_range(tok[3], r.m) || !parse_range(tok[4], r.n) || !parse_range(tok[5], r.k) ||
        !parse_range(tok[6], r.batch))
      return lineno;
    r.variant = variant_by_name(tok[7].c_str());
    if (r.variant < 0) return lineno;
    t.push_back(r);
  }
  return 0;
}

}  // namespace

const char* gemm_variant_name(int v) { return (v >= 0 && v < kVariantCount) ? kVariantNames[v] : nullptr; }

int select_gemm_variant(const GemmProblem& p) {
  if (t_hint != kVariantAuto) return t_hint;
  const int forced = g_forced.load(std::memory_order_relaxed);
  if (forced != kVariantAuto) return forced;
  std::shared_ptr<const Table> t;
  {
    std::lock_guard<std::mutex> lk(g_table_mu);
    t = g_table;
  }
  if (!t) return kVariantAuto;
  for (const Rule& r : *t) {
    if (r.dtype >= 0 && r.dtype != p.dtype) continue;
    if (r.transA >= 0 && r.transA != static_cast<int>(p.transA)) continue;
    if (r.transB >= 0 && r.transB != static_cast<int>(p.transB)) continue;
    if (r.m.has(p.M) && r.n.has(p.N) && r.k.has(p.K) && r.batch.has(p.batch)) return r.variant;
  }
  return kVariantAuto;
}

}  // namespace cuopx

using namespace cuopx;

extern "C" {

int cuopx_tuning_load(const char* text) {
  if (!text) return CUOPX_INVALID_ARGUMENT;
  auto t = std::make_shared<Table>();
  if (parse_table(text, *t) != 0) return CUOPX_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lk(g_table_mu);
  g_table = std::move(t);
  return CUOPX_SUCCESS;
}

int cuopx_tuning_load_file(const char* path) {
  if (!path) return CUOPX_INVALID_ARGUMENT;
  std::ifstream f(path);
  if (!f) return CUOPX_INVALID_ARGUMENT;
  std::stringstream ss;
  ss << f.rdbuf();
  return cuopx_tuning_load(ss.str().c_str());
}

int cuopx_tuning_clear(void) {
  std::lock_guard<std::mutex> lk(g_table_mu);
  g_table.reset();
  return CUOPX_SUCCESS;
}

int cuopx_tuning_rows(void) {
  std::lock_guard<std::mutex> lk(g_table_mu);
  return g_table ? static_cast<int>(g_table->size()) : 0;
}

int cuopx_set_gemm_variant(const char* name) {
  const int v = name ? variant_by_name(name) : kVariantAuto;
  if (v < 0) return CUOPX_INVALID_ARGUMENT;
  g_forced.store(v);
  return CUOPX_SUCCESS;
}

const char* cuopx_gemm_variant_name(int index) { return gemm_variant_name(index); }

int cuopx_set_gemm_variant_thread(const char* name) {
  const int v = name ? variant_by_name(name) : kVariantAuto;
  if (v < 0) return CUOPX_INVALID_ARGUMENT;
  t_hint = v;
  return CUOPX_SUCCESS;
}

}  // extern "C"
