// Per-kernel timestamps of a traced decode step (host and device visible).
#pragma once

namespace smallm {

// One slot per kernel of a traced step (%globaltimer, ns): earliest CTA
// start, earliest CTA past its dependency wait, latest CTA end, and a kind
// code the host assigns.  The production graph passes null slots.
struct TraceSlot {
    unsigned long long t_start, t_ready, t_end, kind;
};

}  // namespace smallm
