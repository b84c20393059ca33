// sw_wavefront.cu -- fast value+marginals path (register/shared-memory wavefront).
// Placeholder until the optimized kernel lands: it declines every shape so the
// plane engine (sw_plane.cu) runs.
#include "sw_internal.h"

namespace d2pb {

size_t wavefront_workspace_bytes(int, int, int, int) { return 0; }

int launch_wavefront(const SwArgs&, int, size_t, cudaStream_t) { return -1; }

}  // namespace d2pb
