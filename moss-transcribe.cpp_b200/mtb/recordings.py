"""Many recordings on one node: partition across GPUs, groups per launch.

A single recording's decode does not shard (its verify steps are sequential
and the 0.6B decoder fits one GPU), so a node decodes independent recordings
side by side: recording i goes to GPU i mod G (round robin, no inter-GPU
communication), and each GPU steps its recordings in groups of up to eight,
one persistent launch per group step (mtb_spec_step_group_async).  The
reference decodes one recording at a time; this is the serving layer around
its strict speculative generate (src/cpu_speculative.cpp:68-147), with every
recording's ids and counters exactly those of its own single-stream decode.

Two ways to spread the GPUs: one process per GPU (torchrun: `partition` by
rank) or one process driving every GPU with one host thread each
(`run_on_devices`).  A worker that raises does not stop the others: their
results are kept and the failure is reported with the device it happened on.
"""
from __future__ import annotations

import threading
from dataclasses import dataclass, field

GROUP_MAX = 8  # decoders verified together in one persistent launch


def partition(n_recordings: int, n_gpus: int, rank: int) -> list[int]:
    """Recordings of GPU `rank`: i with i mod n_gpus == rank, in order."""
    if n_gpus < 1 or not 0 <= rank < n_gpus or n_recordings < 0:
        raise ValueError("need n_gpus >= 1, 0 <= rank < n_gpus, n_recordings >= 0")
    return list(range(rank, n_recordings, n_gpus))


def groups_of(items: list, size: int = GROUP_MAX) -> list[list]:
    """Consecutive groups of at most `size` (one launch per group step)."""
    if size < 1:
        raise ValueError("group size must be >= 1")
    return [items[i:i + size] for i in range(0, len(items), size)]


@dataclass
class Recording:
    """One recording's fused prompt rows [seq][hidden] and decode budget."""
    rows: object
    max_new: int
    eos: int = -1


def decode_recordings(model, recordings: list[Recording], kv_type=None, k_max: int = 8, n_min: int = 3,
                      n_max: int = 3, group_size: int = GROUP_MAX):
    """Decode recordings on `model`'s GPU in groups of `group_size`: each
    member prefilled (mtb_spec_prime), then group steps until all stopped
    (mtb_spec_run_group).  One set of decoders, sized for the largest
    recording, serves every group (priming resets a decoder), so the caches
    and step graphs are made once per GPU, not once per group.  Returns
    [(ids, counters)] in input order."""
    from . import capi
    kv_type = capi.KV_F16 if kv_type is None else kv_type
    recordings = list(recordings)
    if not recordings:
        return []
    max_seq = max(r.rows.shape[0] + r.max_new for r in recordings) + 64
    max_new = max(r.max_new for r in recordings)
    out = []
    pool = []
    try:
        for _ in range(min(group_size, len(recordings))):
            pool.append(capi.Decoder(model, max_seq, kv_type, max_new=max_new))
        for group in groups_of(recordings, group_size):
            decs = pool[:len(group)]
            for d, r in zip(decs, group):
                d.spec_prime(r.rows, r.max_new, r.eos, k_max=k_max, n_min=n_min, n_max=n_max)
            capi.spec_run_group(decs)
            out.extend(d.read_ids() for d in decs)
    finally:
        for d in pool:
            d.close()
    return out


@dataclass
class DeviceFailure:
    device: int
    error: BaseException


@dataclass
class NodeResult:
    results: dict = field(default_factory=dict)   # recording index -> worker result
    failures: list = field(default_factory=list)  # DeviceFailure per failed worker

    def raise_failures(self):
        if self.failures:
            f = self.failures[0]
            raise RuntimeError(f"recording worker on GPU {f.device} failed: {f.error!r} "
                               f"({len(self.failures)} of the node's workers failed)") from f.error


def run_on_devices(n_recordings: int, devices: list[int], worker) -> NodeResult:
    """One host thread per device: `worker(device, indices)` decodes the
    recordings `indices` (this device's round-robin share) and returns
    {index: result}.  Every worker runs to its own end; failures are collected
    (NodeResult.failures), the other devices' results are kept."""
    res = NodeResult()
    lock = threading.Lock()

    def body(rank: int, dev: int):
        mine = partition(n_recordings, len(devices), rank)
        try:
            got = worker(dev, mine)
            with lock:
                res.results.update(got)
        except BaseException as e:  # surfaced to the caller, the other threads go on
            with lock:
                res.failures.append(DeviceFailure(dev, e))

    threads = [threading.Thread(target=body, args=(r, d), name=f"mtb-gpu{d}") for r, d in enumerate(devices)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    return res
