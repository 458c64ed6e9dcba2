// Named NVTX ranges around the library's operator stages, so that a
// profiler's timeline (nsys, ncu's NVTX filters) shows which operator and
// stage each kernel belongs to.  Without a profiler attached the calls do
// nothing measurable.  Host code only.
#pragma once
#include <nvtx3/nvToolsExt.h>

namespace ornith {

class NvtxRange {
  public:
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

}  // namespace ornith
