// awa_profile.cpp -- opt-in per-launch device timing of the library's kernels
// (CUDA events recorded on each launch's stream), reported as
// "profile name=<kernel> launches=<n> ms=<total>" lines.
#include "awa_b200.h"
#include "awa_internal.h"

#include <atomic>
#include <cstdio>
#include <map>
#include <mutex>
#include <string>
#include <vector>

namespace
{

std::atomic<bool> g_enabled{false};
std::mutex g_mutex;
struct Pending
{
    std::string name;
    cudaEvent_t start;
    cudaEvent_t stop;
};
std::vector<Pending> g_pending;
std::vector<cudaEvent_t> g_free;
std::map<std::string, std::pair<long long, double>> g_totals;  // name -> (launches, ms)

}  // namespace

namespace awa
{

bool profiling_enabled()
{
    return g_enabled.load(std::memory_order_relaxed);
}

cudaEvent_t profile_event()
{
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!g_free.empty())
    {
        cudaEvent_t e = g_free.back();
        g_free.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess)
        return nullptr;
    return e;
}

void profile_record(const char* name, cudaEvent_t start, cudaEvent_t stop)
{
    std::lock_guard<std::mutex> lock(g_mutex);
    g_pending.push_back({name, start, stop});
}

}  // namespace awa

extern "C" {

void awa_profile_enable(int enabled)
{
    g_enabled.store(enabled != 0);
}

void awa_profile_reset(void)
{
    std::lock_guard<std::mutex> lock(g_mutex);
    for (Pending& p : g_pending)
    {
        cudaEventSynchronize(p.stop);
        g_free.push_back(p.start);
        g_free.push_back(p.stop);
    }
    g_pending.clear();
    g_totals.clear();
}

int awa_profile_collect(char* buffer, size_t capacity)
{
    std::lock_guard<std::mutex> lock(g_mutex);
    for (Pending& p : g_pending)
    {
        float ms = 0.f;
        if (cudaEventSynchronize(p.stop) == cudaSuccess && cudaEventElapsedTime(&ms, p.start, p.stop) == cudaSuccess)
        {
            auto& entry = g_totals[p.name];
            entry.first += 1;
            entry.second += ms;
        }
        g_free.push_back(p.start);
        g_free.push_back(p.stop);
    }
    g_pending.clear();
    std::string out;
    char line[256];
    for (const auto& kv : g_totals)
    {
        std::snprintf(line, sizeof(line), "profile name=%s launches=%lld ms=%.6f\n", kv.first.c_str(),
                      kv.second.first, kv.second.second);
        out += line;
    }
    if (buffer && capacity)
    {
        const size_t n = out.size() < capacity - 1 ? out.size() : capacity - 1;
        out.copy(buffer, n);
        buffer[n] = 0;
    }
    return (int)out.size();
}

}  // extern "C"
