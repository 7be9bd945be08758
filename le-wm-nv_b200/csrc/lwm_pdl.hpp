// lwm_pdl.hpp — the launching thread's switch for programmatic dependent
// launch (launch_pdl in lwm_device.cuh): on while a PdlScope is open.
#pragma once

namespace lwm {

inline thread_local bool g_pdl_launch = false;

struct PdlScope {
    bool prev;
    PdlScope() : prev(g_pdl_launch) { g_pdl_launch = true; }
    ~PdlScope() { g_pdl_launch = prev; }
    PdlScope(const PdlScope&) = delete;
    PdlScope& operator=(const PdlScope&) = delete;
};

}  // namespace lwm
