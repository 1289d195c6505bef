// spm_sweep_plan: the ring schedule of a host-to-HBM sweep (sweep_ring.h)
// driven by a script of next/rewind calls against a recording backend, on
// the host.  The log it returns is what the CUDA backend of sweep.cu would do
// for the same calls, so the ordering rules (every launch after its copy,
// every overwrite after the overwritten stream's kernel) can be checked
// without a device.
#include "abi.h"
#include "sweep_ring.h"

using namespace spm;

namespace {

struct Recorder final : RingBackend {
    std::vector<int64_t> log;
    int events = 0;
    void put(int64_t kind, int64_t stream, int64_t off, int64_t ev) {
        log.insert(log.end(), {kind, stream, off, ev});
    }
    int create_events() override {
        put(SPM_PLAN_EVENTS, -1, -1, events);
        return events++;
    }
    void wait_consumed(int ev) override { put(SPM_PLAN_WAIT, -1, -1, ev); }
    void copy(uint32_t stream, uint64_t off, int ev) override { put(SPM_PLAN_COPY, stream, int64_t(off), ev); }
    void launch(uint32_t stream, uint64_t off, int ev) override { put(SPM_PLAN_LAUNCH, stream, int64_t(off), ev); }
};

}  // namespace

spm_status spm_sweep_plan(const uint64_t* region_bytes, int32_t streams, uint64_t device_bytes,
                          const int32_t* script, int32_t script_len, int64_t* log, int64_t log_cap,
                          int64_t* log_len) {
    return guarded([&] {
        if (streams <= 0 || !region_bytes) fail(SPM_E_ARG, "parameter stream declares no operations");
        if (script_len < 0 || (script_len && !script) || !log_len) fail(SPM_E_ARG, "bad script");
        std::vector<uint64_t> bytes(region_bytes, region_bytes + streams);
        for (uint64_t b : bytes)
            if (b % 256 || b > device_bytes) fail(SPM_E_ARG, "regions must be 256-byte multiples that fit the ring");
        SweepRing ring(bytes, device_bytes);
        Recorder rec;
        ring.prefetch(rec);
        for (int32_t i = 0; i < script_len; ++i) {
            if (script[i] == SPM_PLAN_NEXT) {
                if (ring.position() >= ring.streams())
                    rec.put(SPM_PLAN_REFUSED, -1, -1, -1);
                else
                    ring.run(rec);
            } else if (script[i] == SPM_PLAN_REWIND) {
                rec.put(SPM_PLAN_REWOUND, -1, -1, -1);
                ring.rewind(rec);
            } else {
                fail(SPM_E_ARG, "unknown script command");
            }
        }
        *log_len = int64_t(rec.log.size() / 4);
        if (log) {
            if (log_cap < *log_len) fail(SPM_E_ARG, "log capacity too small");
            std::copy(rec.log.begin(), rec.log.end(), log);
        }
    });
}
