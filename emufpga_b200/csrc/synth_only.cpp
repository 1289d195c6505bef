// libspmsynth.so: the seeded synthetic-model writer on its own (the encoders
// and GGUF writer of host_synth.cpp, with the format code of host_format.cpp
// they need), with no device code and no CUDA runtime.  A process that must
// not load the GPU engine -- the benchmark's CPU reference arm -- makes its
// input model with it; the bytes are the ones libspmgpu.so's spm_synth_gguf
// writes for the same spec.
#include <cstdlib>

#include "abi.h"

namespace spm {
const std::string& last_error();
}

extern "C" {

const char* spm_last_error(void) { return spm::last_error().c_str(); }
void spm_free(void* p) { std::free(p); }

spm_status spm_synth_gguf(const spm_synth_spec* spec, uint8_t** out, uint64_t* len) {
    return spm::guarded([&] {
        if (!spec || !out || !len) spm::fail(SPM_E_ARG, "null argument");
        *out = spm::synth_gguf(*spec, len);
    });
}

}  // extern "C"
