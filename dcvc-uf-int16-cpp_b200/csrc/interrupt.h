// Process-wide cancellation flag (the reference's uf::ProcessInterrupt,
// include/uf/process.hpp:66-79, src/process.cpp:192-195): a caller sets it
// (from a signal handler or another thread); codec calls check it between
// packets and frames and unwind with "UF operation interrupted".
#pragma once

#include <stdexcept>

namespace ufb {

struct Interrupted : std::runtime_error {
    Interrupted() : std::runtime_error("UF operation interrupted") {}
};

void set_interrupt(bool on);
bool interrupt_requested();
inline void check_interrupt() {
    if (interrupt_requested()) throw Interrupted();
}

}  // namespace ufb
