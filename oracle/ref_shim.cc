// C wrapper over the reference's own index/geometry code (compiled from the
// reference tree by oracle/build_oracle.py). TEST INFRASTRUCTURE ONLY: it lets
// the tests pin this repository's ring/global cache arithmetic and geometry
// validation against native/hyperion_mlx/src/{kv.cc,geometry.cc}.
#include "kv.h"
#include "geometry.h"

#include <cstdint>
#include <cstdio>
#include <string>

using hyperion::model::GlobalCacheIndex;
using hyperion::model::LocalRingIndex;

extern "C" {

// Commit `n_commits` chunks (sizes in `commits`) into a ring of window/gamma and
// report the slot of every position in [0, n_pos) plus the final committed length.
std::uint32_t ref_ring_slots(std::uint32_t window, std::uint32_t gamma,
                             const std::uint32_t* commits, int n_commits,
                             std::uint32_t* slots, std::uint32_t n_pos) {
    LocalRingIndex ring(window, gamma);
    for (int i = 0; i < n_commits; ++i) ring.commit(commits[i]);
    for (std::uint32_t p = 0; p < n_pos; ++p) slots[p] = ring.slot_for(p);
    return ring.committed_len();
}

std::uint32_t ref_ring_capacity(std::uint32_t window, std::uint32_t gamma) {
    return LocalRingIndex(window, gamma).capacity();
}

// Append chunks to a 256-step global index; capacities[i] is the capacity after
// append i.
void ref_global_capacities(std::uint32_t step, const std::uint32_t* appends, int n,
                           std::uint32_t* capacities) {
    GlobalCacheIndex g(step);
    for (int i = 0; i < n; ++i) {
        g.append(appends[i]);
        capacities[i] = g.capacity();
    }
}

// 0 = valid; 1 = from_abi rejected; 2 = validate rejected. Message copied out.
int ref_geometry_check(const HypGeometryParams* p, char* msg, std::size_t len) {
    hyperion::model::Geometry g;
    if (auto e = hyperion::model::Geometry::from_abi(*p, g)) {
        std::snprintf(msg, len, "%s", e->c_str());
        return 1;
    }
    if (auto e = g.validate()) {
        std::snprintf(msg, len, "%s", e->c_str());
        return 2;
    }
    if (len) msg[0] = '\0';
    return 0;
}

}  // extern "C"
