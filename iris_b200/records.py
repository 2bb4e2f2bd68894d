"""Canonical checkpoint records of the teacher-forced chain's stages.

The reference commits each stage's outputs through Raster encodings
(crates/inference/artifacts/src/checkpoint.rs:32-204,
crates/inference/staged/src/artifact_io.rs:46-58); the Raster crate is not
available to this build, so those commitments cannot be reproduced. This
module defines a documented substitute that pins the same content: a stage's
output rows and its own K/V rows, byte for byte, under SHA-256, as a
two-level hash so that the device can hash the rows where they live.

Record layout (all integers little-endian; the digest is the SHA-256 of the
record):

    b"IRISREC2"
    u32 len(stage), stage name (UTF-8)      e.g. "layer_mistral/3"
    u32 start_position, u32 rows, u32 width, u32 kv_width (0 when none)
    u32 leaf                                 bytes a leaf (4096)
    leaf digests of the rows x width int32 (the stage's output activations),
    then of the K rows, then of the V rows (rows x kv_width int32 each):
    SHA-256 of each consecutive `leaf`-byte piece of the array, the last
    piece shorter.

`chain_records` runs a claim's teacher-forced pass stage by stage on the
device and returns each stage's record digest: mistral-dense through
`iris_mistral_layer_range` per range and layer, K/V carried across ranges
(mistral/stage.rs:172-226); gemma-dense through `iris_gemma_layer_range`,
with the range's PLE rows, the carried K/V pruned to each layer's window as
the reference hands it on (prefill_range.rs:82-172, 849-860) and a sharing
layer attending over its donor's keys of the same range.
"""
from __future__ import annotations

import hashlib
import struct
from typing import List, Optional, Sequence, Tuple

import numpy as np

MAGIC = b"IRISREC2"
LEAF = 4096


def _checked(rows, k, v):
    rows = np.ascontiguousarray(rows, "<i4")
    if rows.ndim != 2:
        raise ValueError("rows must be [n][width]")
    if k is not None:
        k = np.ascontiguousarray(k, "<i4")
        v = np.ascontiguousarray(v, "<i4")
        if k.shape != v.shape or k.ndim != 2 or k.shape[0] != rows.shape[0]:
            raise ValueError("K and V must hold one row per output row")
    return rows, k, v


def leaf_digests(a: np.ndarray, leaf: int = LEAF) -> bytes:
    """SHA-256 of each consecutive `leaf`-byte piece of the array's bytes."""
    b = memoryview(np.ascontiguousarray(a)).cast("B")
    return b"".join(hashlib.sha256(b[i:i + leaf]).digest() for i in range(0, len(b), leaf))


def record_header(stage: str, start: int, n: int, width: int, kv_width: int, leaf: int = LEAF) -> bytes:
    name = stage.encode()
    return MAGIC + struct.pack("<I", len(name)) + name + struct.pack("<IIIII", start, n, width, kv_width, leaf)


def stage_record(stage: str, start: int, rows: np.ndarray, k: Optional[np.ndarray] = None,
                 v: Optional[np.ndarray] = None, leaf: int = LEAF) -> bytes:
    rows, k, v = _checked(rows, k, v)
    out = [record_header(stage, start, rows.shape[0], rows.shape[1], 0 if k is None else k.shape[1], leaf),
           leaf_digests(rows, leaf)]
    if k is not None:
        out += [leaf_digests(k, leaf), leaf_digests(v, leaf)]
    return b"".join(out)


def stage_digest(stage: str, start: int, rows: np.ndarray, k=None, v=None, leaf: int = LEAF) -> str:
    """SHA-256 of the stage's record."""
    return hashlib.sha256(stage_record(stage, start, rows, k, v, leaf)).hexdigest()


def digest_from_leaves(stage: str, start: int, n: int, width: int, kv_width: int, leaves: bytes,
                       leaf: int = LEAF) -> str:
    """The record digest from leaf digests computed elsewhere (the device's)."""
    return hashlib.sha256(record_header(stage, start, n, width, kv_width, leaf) + leaves).hexdigest()


def leaf_count(nbytes: int, leaf: int = LEAF) -> int:
    return (nbytes + leaf - 1) // leaf


def window_start(position: int, window: int) -> int:
    """prefill_range.rs:866-874: the first position a query at `position` sees."""
    return 0 if window == 0 else max(0, position + 1 - window)


def output_kv(carried, own_k, own_v, start: int, window: int):
    """prefill_range.rs:849-860: the keys a range hands on, (positions, k, v):
    the carried keys the window still holds for the range's first position,
    then the range's own."""
    pos, k, v = carried
    keep = pos >= window_start(start, window)
    n = own_k.shape[0]
    return (np.concatenate([pos[keep], np.arange(start, start + n, dtype=np.uint32)]),
            np.concatenate([k[keep], own_k]), np.concatenate([v[keep], own_v]))


def chain_records(model, ids: Sequence[int], range_size: int = 512) -> List[Tuple[str, int, str]]:
    """(stage, start_position, SHA-256 of its record) for every (range, layer)
    stage of a claim whose prompt-and-output token ids are `ids`, ranges of
    `range_size` rows. `model` offers embed / layer_range (mistral-dense) or
    embed / ple_rows / gemma_layer_range (gemma-dense)."""
    if model.cfg.family == "gemma":
        return _gemma_chain_records(model, ids, range_size)
    cfg = model.cfg
    kvd = cfg.kv_heads * cfg.head_dim
    carried_k = [np.zeros((0, kvd), np.int32) for _ in range(cfg.layers)]
    carried_v = [np.zeros((0, kvd), np.int32) for _ in range(cfg.layers)]
    out = []
    for start in range(0, len(ids), range_size):
        rows = model.embed(ids[start:start + range_size])
        for layer in range(cfg.layers):
            rows, own_k, own_v = model.layer_range(layer, rows, start, carried_k[layer], carried_v[layer])
            out.append((f"layer_mistral/{layer}", start, stage_digest(f"layer_mistral/{layer}", start, rows,
                                                                       own_k, own_v)))
            carried_k[layer] = np.concatenate([carried_k[layer], own_k])
            carried_v[layer] = np.concatenate([carried_v[layer], own_v])
    return out


def _gemma_chain_records(model, ids, range_size):
    cfg = model.cfg
    kvd = cfg.kv_heads * cfg.head_dim
    empty = (np.zeros(0, np.uint32), np.zeros((0, kvd), np.int32), np.zeros((0, kvd), np.int32))
    carried = [empty] * cfg.layers
    out = []
    for start in range(0, len(ids), range_size):
        part = ids[start:start + range_size]
        rows = model.embed(part)
        ple = model.ple_rows(part)
        handed = []
        for layer in range(cfg.layers):
            donor = cfg.kv_donor(layer)
            rows, own_k, own_v = model.gemma_layer_range(layer, rows, start, ple[:, layer],
                                                         prior=carried[layer],
                                                         donor=handed[donor] if donor >= 0 else None)
            name = f"prefill_range/{layer}"
            out.append((name, start, stage_digest(name, start, rows, own_k, own_v)))
            handed.append(output_kv(carried[layer], own_k, own_v, start, cfg.window(layer)))
        carried = handed
    return out


class _Pinned:
    """A page-locked host array from iris_host_alloc."""

    def __init__(self, shape, dtype=np.int32):
        import ctypes as C
        from . import _lib
        n = int(np.prod(shape))
        dtype = np.dtype(dtype)
        self._p = C.c_void_p()
        _lib.check(_lib.lib().iris_host_alloc(n * dtype.itemsize, C.byref(self._p)), "iris_host_alloc")
        ctype = {np.dtype(np.int32): C.c_int32, np.dtype(np.uint8): C.c_uint8}[dtype]
        self.a = np.ctypeslib.as_array(C.cast(self._p, C.POINTER(ctype)), shape=(n,)).reshape(shape)

    @property
    def ptr(self):
        return self._p

    def free(self):
        from . import _lib
        if self._p:
            _lib.lib().iris_host_free(self._p)
            self._p = None


def chain_claim(session, ids: Sequence[int], range_size: int = 512, slots: int = 12,
                workers: Optional[int] = None, device_hash: bool = True):
    """A claim's teacher-forced pass range by range on a session, every stage's
    record digest taken while the device runs the next stages. With
    `device_hash` the device hashes each stage's rows and own K/V into the
    record's leaf digests (iris_session_range_layer_leaves) and a worker
    thread waits for them (iris_session_ticket_wait) and takes the record's
    digest from the leaves; otherwise the rows and K/V are copied out and
    hashed on the host. Either way the digest is stage_digest's. `slots`
    page-locked buffer sets are in flight at most. After each range the head
    check selects a token for every row. Returns (records [(stage, start,
    digest)], selected token ids, their scores)."""
    import ctypes as C
    import os
    from concurrent.futures import ThreadPoolExecutor
    from . import _lib
    L = _lib.lib()
    if not workers and device_hash:
        # the host only hashes a short header and the leaves (~96 KB a stage):
        # two threads keep up, and a wide pool of threads waking on tickets
        # was seen to stall the issuing thread (641 against 357 ms a claim)
        workers = 2
    elif not workers:  # the host cores this process may use, shared with the node's other ranks
        cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
        workers = max(1, cores // max(1, int(os.environ.get("LOCAL_WORLD_SIZE", "1"))))
    model = session.model
    cfg = model.cfg
    if not 0 < range_size <= 512:
        raise ValueError("ranges hold 1 to 512 rows")
    kvd = cfg.kv_heads * cfg.head_dim
    stage_name = "prefill_range" if cfg.family == "gemma" else "layer_mistral"
    if device_hash:  # a range's layers are issued in batches of up to 32 (a session keeps 64 tickets)
        batch = min(cfg.layers, 32)
        slots = max(slots, 2 * batch)
    # page-locked buffer sets, kept on the session for its next claims (pinning
    # host pages can take long; Session.close frees them)
    cache = session.__dict__.setdefault("_pinned_sets", {})
    key = (device_hash, range_size, slots)
    sets = cache.get(key)
    if sets is None:
        if device_hash:
            nleaves = leaf_count(range_size * cfg.hidden * 4) + 2 * leaf_count(range_size * kvd * 4)
            sets = [(_Pinned((nleaves * 32,), np.uint8),) for _ in range(slots)]
        else:
            sets = [(_Pinned((range_size, cfg.hidden)), _Pinned((range_size, kvd)), _Pinned((range_size, kvd)))
                    for _ in range(slots)]
        cache[key] = sets
    busy = [None] * slots
    ids = np.ascontiguousarray(ids, np.uint32)
    selected = np.empty(len(ids), np.uint32)
    scores = np.empty(len(ids), np.int32)
    jobs = []

    def digest(slot, ticket, name, start, n):
        _lib.check(L.iris_session_ticket_wait(session.handle, ticket), "iris_session_ticket_wait")
        if device_hash:
            count = leaf_count(n * cfg.hidden * 4) + 2 * leaf_count(n * kvd * 4)
            return name, start, digest_from_leaves(name, start, n, cfg.hidden, kvd, sets[slot][0].a[:count * 32].tobytes())
        r, k, v = sets[slot]
        return name, start, stage_digest(name, start, r.a[:n], k.a[:n], v.a[:n])

    with ThreadPoolExecutor(max_workers=workers) as pool:
        j, base = 0, session.length
        for start in range(base, base + len(ids), range_size):
            off = start - base
            part = ids[off:off + range_size]
            n = len(part)
            _lib.check(L.iris_session_range_begin(session.handle, _lib.ptr(part, C.c_uint32), n),
                       "iris_session_range_begin")
            if device_hash:
                for first in range(0, cfg.layers, batch):
                    cnt = min(batch, cfg.layers - first)
                    use = [(j + i) % slots for i in range(cnt)]
                    for slot in use:
                        if busy[slot] is not None:
                            busy[slot].result()  # the set's previous record is hashed
                    ptrs = (C.c_void_p * cnt)(*[sets[slot][0].ptr for slot in use])
                    tickets = (C.c_uint32 * cnt)()
                    _lib.check(L.iris_session_range_layers_leaves(session.handle, cnt, LEAF, ptrs, tickets),
                               "iris_session_range_layers_leaves")
                    for i, slot in enumerate(use):
                        busy[slot] = pool.submit(digest, slot, tickets[i], f"{stage_name}/{first + i}", start, n)
                        jobs.append(busy[slot])
                    j += cnt
            else:
                for layer in range(cfg.layers):
                    slot = j % slots
                    if busy[slot] is not None:
                        busy[slot].result()  # the set's previous record is hashed
                    ticket = C.c_uint32()
                    r, k, v = sets[slot]
                    _lib.check(L.iris_session_range_layer(session.handle, layer, r.ptr, k.ptr, v.ptr,
                                                          C.byref(ticket)), "iris_session_range_layer")
                    busy[slot] = pool.submit(digest, slot, ticket.value, f"{stage_name}/{layer}", start, n)
                    jobs.append(busy[slot])
                    j += 1
            _lib.check(L.iris_session_range_end(session.handle, _lib.ptr(selected[off:off + n], C.c_uint32),
                                                _lib.ptr(scores[off:off + n], C.c_int32)),
                       "iris_session_range_end")
        records = [f.result() for f in jobs]
    return records, selected, scores
