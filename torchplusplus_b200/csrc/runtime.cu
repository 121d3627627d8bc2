// Library-level plumbing of the C-ABI: error messages, version, launch count.
#include <atomic>
#include <cstdlib>
#include "common.cuh"

namespace tpp {

static thread_local std::string g_last_error;
static std::atomic<uint64_t> g_launches{0};

static thread_local int g_sm_budget = 0;

void set_error(const std::string& msg) { g_last_error = msg; }
int sm_budget() {
  const int n = num_sms();
  return g_sm_budget > 0 && g_sm_budget < n ? g_sm_budget : n;
}
void count_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("TPP_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return TPP_ERR_LAUNCH;
  }
  count_launch();
  return TPP_OK;
}

}  // namespace tpp

extern "C" const char* tpp_last_error(void) { return tpp::g_last_error.c_str(); }
extern "C" const char* tpp_version(void) { return "tpp_b200 0.1 (sm_100a)"; }
extern "C" uint64_t tpp_launch_count(void) { return tpp::g_launches.load(); }
extern "C" int tpp_set_sm_budget(int sms) {
  if (sms < 0) {
    tpp::set_error("tpp_set_sm_budget: sms must be >= 0 (0 = the whole device)");
    return TPP_ERR_SHAPE;
  }
  tpp::g_sm_budget = sms;
  return TPP_OK;
}
