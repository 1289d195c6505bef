// The ring schedule of a host-to-HBM sweep (sweep.cu), kept apart from CUDA
// so that the same code can be run against a recording backend and checked
// on the host (spm_sweep_plan).
//
// Streams run in file order, cyclically: sequence position s runs stream
// s % n.  Each copied stream occupies one region of a device ring of `cap`
// bytes; regions start 256-byte aligned, go forward from the end of the last
// one and wrap to 0 when the end does not fit.  A region may be overwritten
// only once the kernel that reads its occupant has been enqueued: the copy
// then waits (on the device) for that kernel's `consumed` event.  Each
// occupant holds its own event pair until it is overwritten or dropped, so
// an event is never re-recorded while a wait on its previous record is still
// to be enqueued.
#pragma once
#include <cstdint>
#include <deque>
#include <stdexcept>
#include <vector>

namespace spm {

struct RingOccupant {
    uint64_t seq = 0, off = 0, bytes = 0;
    bool launched = false;
    int ev = -1;
};

// What the schedule asks of the device.
struct RingBackend {
    virtual ~RingBackend() = default;
    virtual int create_events() = 0;                          // a new (copied, consumed) pair; returns its index
    virtual void wait_consumed(int ev) = 0;                   // the copy stream waits for consumed[ev]
    virtual void copy(uint32_t stream, uint64_t off, int ev) = 0;  // copy the stream to off, then record copied[ev]
    virtual void launch(uint32_t stream, uint64_t off, int ev) = 0;  // wait copied[ev], run, record consumed[ev]
};

class SweepRing {
  public:
    SweepRing(std::vector<uint64_t> region_bytes, uint64_t cap) : bytes_(std::move(region_bytes)), cap_(cap) {}

    uint64_t streams() const { return bytes_.size(); }
    uint64_t position() const { return run_seq_ - sweep_start_; }
    uint64_t copies() const { return copies_; }
    const std::deque<RingOccupant>& live() const { return live_; }

    // Read ahead as far as the ring allows, at most one sweep beyond the
    // next stream to run.
    void prefetch(RingBackend& be) {
        const uint64_t n = bytes_.size();
        while (copy_seq_ < run_seq_ + n && try_copy(be)) {
        }
    }

    // Run the next stream: copy it first if it is not in the ring yet (this
    // always succeeds: every live occupant has been launched), launch it,
    // then read ahead.  Returns the stream index; the caller checks the
    // position against the stream count before.
    uint32_t run(RingBackend& be) {
        const uint64_t n = bytes_.size();
        if (copy_seq_ == run_seq_) try_copy(be);
        RingOccupant* o = nullptr;
        for (RingOccupant& c : live_)
            if (c.seq == run_seq_) o = &c;
        if (!o) throw std::logic_error("sweep ring: the next stream is not in the ring");
        const uint32_t stream = uint32_t(run_seq_ % n);
        be.launch(stream, o->off, o->ev);
        o->launched = true;
        ++run_seq_;
        prefetch(be);
        return stream;
    }

    // Back to the first stream.  At a sweep boundary what was read ahead is
    // the next sweep's; in mid-sweep it is dropped and the next sweep starts
    // at the next multiple of n.
    void rewind(RingBackend& be) {
        const uint64_t n = bytes_.size();
        const uint64_t pos = position();
        if (pos != 0 && pos != n) {
            for (auto it = live_.begin(); it != live_.end();) {
                if (!it->launched) {
                    free_ev_.push_back(it->ev);
                    it = live_.erase(it);
                } else {
                    ++it;
                }
            }
            copy_seq_ = (copy_seq_ + n - 1) / n * n;
            run_seq_ = copy_seq_;
            prefetch(be);
        }
        sweep_start_ = run_seq_;
    }

  private:
    bool try_copy(RingBackend& be) {
        const uint64_t n = bytes_.size();
        const uint32_t stream = uint32_t(copy_seq_ % n);
        const uint64_t b = bytes_[stream];
        const uint64_t off = head_ + b <= cap_ ? head_ : 0;
        auto overlaps = [&](const RingOccupant& o) { return b && o.bytes && off < o.off + o.bytes && o.off < off + b; };
        for (const RingOccupant& o : live_)
            if (overlaps(o) && !o.launched) return false;
        for (auto it = live_.begin(); it != live_.end();) {
            if (overlaps(*it)) {
                be.wait_consumed(it->ev);
                free_ev_.push_back(it->ev);
                it = live_.erase(it);
            } else {
                ++it;
            }
        }
        RingOccupant o;
        o.seq = copy_seq_;
        o.off = off;
        o.bytes = b;
        if (free_ev_.empty()) {
            o.ev = be.create_events();
        } else {
            o.ev = free_ev_.back();
            free_ev_.pop_back();
        }
        be.copy(stream, off, o.ev);
        live_.push_back(o);
        head_ = off + b;
        ++copy_seq_;
        ++copies_;
        return true;
    }

    std::vector<uint64_t> bytes_;
    uint64_t cap_;
    std::deque<RingOccupant> live_;
    std::vector<int> free_ev_;
    uint64_t head_ = 0, run_seq_ = 0, copy_seq_ = 0, sweep_start_ = 0, copies_ = 0;
};

}  // namespace spm
