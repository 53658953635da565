// Process-wide cancellation flag (declarations in interrupt.h).
#include "interrupt.h"

#include <atomic>

namespace ufb {

namespace {
std::atomic<int> g_interrupt{0};  // lock-free: safe to set from a signal handler
}  // namespace

void set_interrupt(bool on) { g_interrupt.store(on ? 1 : 0, std::memory_order_relaxed); }

bool interrupt_requested() { return g_interrupt.load(std::memory_order_relaxed) != 0; }

}  // namespace ufb
