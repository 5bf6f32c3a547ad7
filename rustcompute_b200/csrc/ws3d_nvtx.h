// ws3d_nvtx.h -- NVTX ranges around the library's phases (upload, slab
// connect, steps, download), so that an Nsight timeline shows them by name.
//
// Categories and colours follow the reference's NVTX profiler
// (ringkernel-cuda/src/profiling/nvtx.rs: NvtxCategory Kernel = 1,
// Transfer = 2, Sync = 4).  NVTX v3 is header-only: with no tool attached a
// range costs one check of an injection pointer; nothing is linked.
#pragma once

#include <nvtx3/nvToolsExt.h>

#include <cstdint>

namespace ws3d {

enum NvtxCategory : uint32_t { kNvtxKernel = 1, kNvtxTransfer = 2, kNvtxSync = 4 };

// Scoped range: pushed on construction, popped on destruction.
class NvtxRange {
   public:
    NvtxRange(const char* name, NvtxCategory cat) {
        nvtxEventAttributes_t a = {};
        a.version = NVTX_VERSION;
        a.size = NVTX_EVENT_ATTRIB_STRUCT_SIZE;
        a.category = cat;
        a.colorType = NVTX_COLOR_ARGB;
        a.color = cat == kNvtxKernel ? 0xFF00B4D8u : cat == kNvtxTransfer ? 0xFF2A9D8Fu
                                                                           : 0xFFE9C46Au;
        a.messageType = NVTX_MESSAGE_TYPE_ASCII;
        a.message.ascii = name;
        nvtxRangePushEx(&a);
    }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

}  // namespace ws3d
