"""Decoder preemption checkpoints: keep generated KV when HBM is reclaimed.

Behaviour of the reference (lmcache_ascend/v1/preemption_checkpoint.py:72-464,
local_checkpoint.py:44-361, checkpoint_writeback.py:37-493; contract in
docs/preemption_checkpoint.md):

* ``capture`` runs synchronously when the scheduler preempts a decoding
  request and is about to reuse its blocks: the KV of positions
  ``[start, end)`` is copied out of the paged cache into CPU chunk objects.
  Captured fragments stay private to the (request, generation) pair.
* ``seal`` arrives once the engine knows the accepted token ids (speculative
  tokens may be rejected): the captured span that the accepted tokens cover
  is published.  Here every chunk key is the prefix hash of its tokens, so
  publication is a store of the fragments under the accepted token chain, and
  a resumed request finds them through the ordinary lookup / retrieve path
  (which also covers tokens stored earlier, e.g. the prompt).  Published
  chunks are ordinary CPU-tier entries: evictable, and written back to slower
  tiers by the storage manager; the write-back of a seal goes through the
  engine's put window (bounded bytes and batches in flight, sticky errors,
  fenced per request as ``ckpt:<req_id>``).
* ``cancel`` drops a generation's private fragments; a newer generation of
  the same request supersedes older ones (stale seals are ignored).
* ``available`` reports how many leading tokens of a request can be restored;
  ``restore`` loads them into the request's new blocks.
"""

from __future__ import annotations

import threading
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from ..utils.logging import init_logger
from .memory_management import MemoryFormat, MemoryObj

logger = init_logger(__name__)


@dataclass
class CheckpointResult:
    req_id: str
    generation: int
    published_tokens: int     # leading tokens restorable after the seal
    stored_chunks: int
    dropped_tokens: int       # captured but not covered by accepted tokens


@dataclass
class _Capture:
    start: int
    end: int
    tokens: torch.Tensor      # token ids of [0, end) at capture time
    chunks: List[Tuple[int, int, MemoryObj]] = field(default_factory=list)


class PreemptionCheckpointer:
    def __init__(self, engine):
        self.engine = engine
        self.chunk_size = engine.config.chunk_size
        self._lock = threading.Lock()
        self._jobs: Dict[Tuple[str, int], _Capture] = {}
        self._latest: Dict[str, int] = {}
        self.results: List[CheckpointResult] = []

    # ------------------------------------------------------------ capture
    @torch.no_grad()
    def capture(self, req_id: str, generation: int, token_ids: Sequence[int],
                slot_mapping: torch.Tensor, start: int = 0, end: Optional[int] = None) -> int:
        """Copy the KV of positions [start, end) out of the paged cache.
        ``slot_mapping`` maps positions 0..end-1 to the request's slots.
        ``start`` is rounded down to a chunk boundary (chunks are the storage
        unit); returns the number of captured tokens."""
        tokens = torch.as_tensor(list(token_ids), dtype=torch.long)
        end = len(tokens) if end is None else min(end, len(tokens))
        start = (max(0, start) // self.chunk_size) * self.chunk_size
        if end <= start:
            return 0
        with self._lock:
            if generation < self._latest.get(req_id, -1):
                logger.warning("stale capture %s gen %d ignored", req_id, generation)
                return 0
            self._drop_older(req_id, generation)
            self._latest[req_id] = generation
        conn = self.engine.gpu_connector
        layout = conn.layout
        fmt = getattr(conn, "memory_format", MemoryFormat.KV_2LTD)
        sm = self.engine.storage_manager
        cap = _Capture(start, end, tokens[:end].clone())
        starts, ends, objs = [], [], []
        for s in range(start, end, self.chunk_size):
            e = min(s + self.chunk_size, end)
            o = sm.allocate(torch.Size(layout.chunk_shape(e - s)), layout.dtype, fmt)
            if o is None:
                for _, _, x in cap.chunks:
                    x.ref_count_down()
                raise MemoryError("preemption checkpoint: out of CPU cache memory")
            cap.chunks.append((s, e, o))
            starts.append(s)
            ends.append(e)
            objs.append(o)
        gen = conn.batched_from_gpu(objs, starts, ends, slot_mapping=slot_mapping, sync=True)
        if gen is not None and hasattr(gen, "__next__"):  # layerwise connector
            raise TypeError("capture needs a whole-chunk GPU connector")
        with self._lock:
            self._jobs[(req_id, generation)] = cap
        return end - start

    # --------------------------------------------------------------- seal
    def seal(self, req_id: str, generation: int, accepted_token_ids: Sequence[int]
             ) -> Optional[CheckpointResult]:
        """Publish the captured span covered by the accepted tokens."""
        with self._lock:
            if generation != self._latest.get(req_id):
                logger.warning("seal %s gen %d: not the latest generation", req_id, generation)
                return None
            cap = self._jobs.pop((req_id, generation), None)
        if cap is None:
            return None
        acc = torch.as_tensor(list(accepted_token_ids), dtype=torch.long)
        n = min(len(acc), cap.end)
        agree = int((acc[:n] == cap.tokens[:n]).to(torch.int8).cumprod(0).sum()) if n else 0
        cs = self.chunk_size
        eng = self.engine
        keys_by_end = {e: k for _, e, k in eng._chunks(acc[:agree])}
        stored, covered = 0, cap.start
        sm = eng.storage_manager
        window = eng.layerwise_put_queue  # bounds the write-back to slower tiers
        for s, e, obj in cap.chunks:
            k = keys_by_end.get(e)
            full = (e - s) == cs or eng.config.save_unfull_chunk
            if e <= agree and k is not None and full and s == covered:
                size = obj.get_size()
                window.admit(size)
                try:
                    futs = sm.batched_put([k], [obj])
                except BaseException as err:
                    window.record_failure(err)
                    raise
                window.submit(size, futs, req_id=f"ckpt:{req_id}", keys=[k])
                stored += 1
                covered = e
            obj.ref_count_down()  # the tier holds its own reference
        res = CheckpointResult(req_id, generation, covered if stored else 0, stored,
                               max(0, cap.end - covered))
        with self._lock:
            self.results.append(res)
        return res

    # ---------------------------------------------------- restore / cancel
    def available(self, token_ids: Sequence[int]) -> int:
        """Leading tokens of ``token_ids`` restorable from the cache."""
        return int(self.engine.lookup(torch.as_tensor(list(token_ids), dtype=torch.long)))

    def restore(self, token_ids: Sequence[int], slot_mapping: torch.Tensor) -> int:
        tokens = torch.as_tensor(list(token_ids), dtype=torch.long)
        n = self.available(tokens)
        if n == 0:
            return 0
        ret = self.engine.retrieve(tokens[:n], slot_mapping=slot_mapping[:n])
        return int(ret.sum())

    def cancel(self, req_id: str, generation: Optional[int] = None) -> None:
        with self._lock:
            gens = [g for (r, g) in self._jobs if r == req_id and (generation is None
                                                                  or g == generation)]
            caps = [self._jobs.pop((req_id, g)) for g in gens]
            if generation is None:
                self._latest.pop(req_id, None)
        for cap in caps:
            for _, _, o in cap.chunks:
                o.ref_count_down()

    def _drop_older(self, req_id: str, generation: int) -> None:
        for (r, g) in [k for k in self._jobs if k[0] == req_id and k[1] < generation]:
            for _, _, o in self._jobs.pop((r, g)).chunks:
                o.ref_count_down()

    def pending(self) -> int:
        with self._lock:
            return len(self._jobs)

    def close(self) -> None:
        with self._lock:
            jobs, self._jobs = list(self._jobs.values()), {}
        for cap in jobs:
            for _, _, o in cap.chunks:
                o.ref_count_down()
