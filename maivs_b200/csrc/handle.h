// The state behind one maivs_index handle, shared by the C ABI sources (capi.cpp, concurrent.cpp).
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "cuda/engine.h"
#include "host/index_host.h"

struct maivs_index {
    maivs::HostIndex h;
    // cell-range sharding (declared before `d`, which points at it, so it is destroyed after)
    std::unique_ptr<maivs::Exchange> exch;
    int shard_rank = 0, shard_world = 1;
    std::unique_ptr<maivs::DeviceIndex> d;
    // shards of the in-process emulation of the sharded protocol
    std::vector<std::unique_ptr<maivs::DeviceIndex>> emu;
    uint64_t emu_version = ~0ull;
    int emu_world = 0, emu_device = -1;
    int device = 0;
    std::string err;
    std::mutex mu;
    // host copies served by maivs_array, rebuilt on demand
    std::map<std::string, std::vector<uint8_t>> arrays;
    uint64_t arrays_version = ~0ull;
};

namespace maivs_capi {
// Makes the handle's device image current (uploads after a mutation); returns a maivs_status and
// leaves the message in ix->err. The caller holds whatever lock guards ix->h.
int device_image(maivs_index* ix);
// Refreshes the host copies that maivs_array serves.
void host_arrays(maivs_index* ix);
}  // namespace maivs_capi
