"""Host logic of the node-level recording scheduler (mtb/recordings.py), on
CPU: the round-robin partition, the groups of one launch, and one host thread
per device where a failing worker is reported with its device while the other
devices' recordings finish."""
import threading

import pytest

from mtb import recordings


def test_partition_round_robin_covers_every_recording_once():
    for n, g in [(64, 1), (64, 2), (64, 8), (10, 3), (3, 8), (0, 4)]:
        parts = [recordings.partition(n, g, r) for r in range(g)]
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(n))
        for r, p in enumerate(parts):
            assert all(i % g == r for i in p)
            assert len(p) in (n // g, n // g + 1)
    with pytest.raises(ValueError):
        recordings.partition(8, 2, 2)


def test_groups_of_eight():
    assert recordings.groups_of(list(range(17))) == [list(range(8)), list(range(8, 16)), [16]]
    assert recordings.groups_of([], 8) == []


def test_one_thread_per_device_and_a_failing_worker():
    seen = {}
    lock = threading.Lock()

    def worker(dev, idx):
        with lock:
            seen[dev] = (threading.current_thread().name, list(idx))
        if dev == 5:
            raise RuntimeError("simulated decode failure")
        return {i: ("ok", dev) for i in idx}

    res = recordings.run_on_devices(20, [3, 5, 7], worker)
    assert seen[3][1] == list(range(0, 20, 3)) and seen[5][1] == list(range(1, 20, 3))
    assert len({name for name, _ in seen.values()}) == 3  # one thread each
    assert sorted(res.results) == sorted(list(range(0, 20, 3)) + list(range(2, 20, 3)))  # the others finished
    assert len(res.failures) == 1 and res.failures[0].device == 5
    with pytest.raises(RuntimeError, match="GPU 5"):
        res.raise_failures()


def test_all_workers_succeed():
    res = recordings.run_on_devices(9, [0, 1], lambda dev, idx: {i: dev for i in idx})
    res.raise_failures()
    assert res.results == {i: i % 2 for i in range(9)}
