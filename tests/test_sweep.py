"""The host-to-HBM sweep on the CPU: its ring schedule and its refusals.

spm_sweep_plan runs the schedule that spm_sweep_next / spm_sweep_rewind
drive on the device (the same SweepRing code) against a recording backend.
The checker below replays each log and asserts the rules the device relies
on: streams run in file order and restart after a rewind; a launch reads the
region its stream was last copied to, with nothing copied over it since;
a copy never lands on a stream that is copied but not yet run; a region is
overwritten only after a wait on the consumed event recorded by the launch
that read it; regions stay inside the ring.
"""
import numpy as np
import pytest

import emufpga_b200 as eb
from emufpga_b200 import spmfile as sf
from emufpga_b200 import sweep as S
from tests.spm_cases import sixteenths


def check(log, regions, cap, script):
    n = len(regions)
    created = set()
    occupants = []          # dicts: stream, off, size, ev, launched, consumed_seq
    last_record = {}        # ev -> id of the launch that last recorded consumed[ev]
    waited = set()          # (ev, launch id) pairs waited on by the copy stream
    launches = 0
    expected = 0            # next stream the sweep should run
    position = 0            # streams run since the last rewind
    at_end = False
    for kind, stream, off, ev in log:
        if kind == S.EVENTS:
            assert ev not in created
            created.add(ev)
        elif kind == S.WAIT:
            assert ev in last_record, "wait on a consumed event nobody recorded"
            waited.add((ev, last_record[ev]))
        elif kind == S.COPY:
            assert ev in created
            size = regions[stream]
            assert 0 <= off and off + size <= cap
            for o in occupants:
                if o["alive"] and o["size"] and size and off < o["off"] + o["size"] and o["off"] < off + size:
                    assert o["launched"], "a copy landed on a stream that has not run"
                    assert (o["ev"], o["launch"]) in waited, "overwrite without waiting for its reader"
                    o["alive"] = False
            occupants.append(dict(stream=stream, off=off, size=size, ev=ev, launched=False, launch=None,
                                  alive=True))
        elif kind == S.LAUNCH:
            assert stream == expected and not at_end
            mine = [o for o in occupants if o["alive"] and not o["launched"] and o["stream"] == stream]
            assert mine, "launch of a stream that was not copied"
            o = mine[0]
            assert (o["off"], o["ev"]) == (off, ev)
            o["launched"] = True
            o["launch"] = launches
            last_record[ev] = launches
            launches += 1
            position += 1
            expected = (expected + 1) % n
            at_end = position == n
        elif kind == S.REFUSED:
            assert at_end
        elif kind == S.REWOUND:
            if 0 < position < n:  # mid-sweep: what was read ahead is dropped
                for o in occupants:
                    if o["alive"] and not o["launched"]:
                        o["alive"] = False
            expected, position, at_end = 0, 0, False
    return launches


@pytest.mark.parametrize("seed", range(40))
def test_random_rings_keep_every_ordering_rule(seed):
    rng = np.random.default_rng(seed)
    n = int(rng.integers(1, 9))
    regions = [256 * int(k) for k in rng.integers(0, 12, n)]
    largest = max(max(regions), 256)
    cap = 256 * int(rng.integers(largest // 256, sum(regions) // 256 + 3))
    script = []
    for _ in range(int(rng.integers(1, 5))):
        stop = int(rng.integers(0, n + 2))  # > n: extra calls at the end are refused
        script += [S.NEXT] * stop + [S.REWIND]
    log = S.plan(regions, cap, script)
    runs = sum(1 for r in log if r[0] == S.LAUNCH)
    assert check(log, regions, cap, script) == runs
    # every NEXT within a sweep ran a stream; the rest were refused
    expected = sum(min(k, n) for k in map(len, "".join("x" if c == S.NEXT else "|" for c in script).split("|")))
    assert runs == expected


def test_a_ring_of_one_stream_serialises_copy_and_run():
    log = S.plan([512, 512, 512], 512, [S.NEXT] * 3 + [S.REWIND] + [S.NEXT] * 3)
    check(log, [512, 512, 512], 512, None)
    kinds = [r[0] for r in log if r[0] in (S.COPY, S.LAUNCH)]
    # copy, launch, copy, launch ...: nothing is read ahead past the one slot
    assert kinds == [S.COPY, S.LAUNCH] * 6 + [S.COPY]


def test_a_ring_that_holds_everything_reads_a_whole_sweep_ahead():
    regions = [256, 512, 768]
    log = S.plan(regions, 4 * sum(regions), [S.NEXT] * 3)
    check(log, regions, 4 * sum(regions), None)
    kinds = [r[0] for r in log if r[0] in (S.COPY, S.LAUNCH)]
    assert kinds[:3] == [S.COPY] * 3  # the whole first sweep is in flight at open
    assert kinds.count(S.COPY) == 6   # and the next sweep's streams by its end


def test_plan_refusals():
    with pytest.raises(eb.SpmError):
        S.plan([], 1024, [S.NEXT])
    with pytest.raises(eb.SpmError):
        S.plan([100], 1024, [S.NEXT])
    with pytest.raises(eb.SpmError):
        S.plan([2048], 1024, [S.NEXT])
    with pytest.raises(eb.SpmError):
        S.plan([256], 1024, [7])


def mixed_file():
    w = sf.SpmWriter([(3, 2, 4)])
    w.write_group(1.0, [1, 0, -1, 1])
    w.write_group(0.5, [-1, 0])
    tern = w.finish()
    dense = sf.dense_stream_bytes(sixteenths(5, 8 * 4), 16)
    return (sf.render_header(2) + sf.render_descriptor(3, 2, 4) + sf.render_descriptor(8, 4, 16, sf.F32)
            + tern[64:] + dense)


def test_open_refusals_need_no_device(tmp_path):
    data = mixed_file()
    with pytest.raises(eb.SpmError) as e:
        S.Sweep(data, device_bytes=100)
    assert e.value.code == -1 and "cannot hold the largest stream" in str(e.value)
    q = sf.SpmWriter([(2, 32, 64, sf.Q8_0)])  # two blocks in one group
    q.write_raw_group(1.0, bytes(sf.bytes_for(sf.Q8_0, 64)), 64)
    with pytest.raises(eb.SpmError, match="unexpected packed group"):
        S.Sweep(q.finish())
    with pytest.raises(eb.SpmError) as e:
        S.Sweep(sf.render_header(0))
    assert e.value.code == -1
    with pytest.raises(eb.SpmError) as e:
        S.Sweep(data[:-1])
    assert e.value.code == -3
    with pytest.raises(eb.SpmError) as e:
        S.Sweep(str(tmp_path / "missing.spm"))
    assert e.value.code == -4


@pytest.mark.skipif(__import__("torch").cuda.is_available(), reason="checks the refusal without a device")
def test_open_without_a_device_fails_loudly(tmp_path):
    path = tmp_path / "mixed.spm"
    path.write_bytes(mixed_file())
    for src in (mixed_file(), str(path)):
        with pytest.raises(eb.SpmError) as e:
            S.Sweep(src)
        assert e.value.code == -10
