"""RemoteFill: a prefiller places a request's KV straight into the decoder's
paged blocks, window by window, under an explicit session protocol with
deadlines, replay, admission limits and a circuit breaker; any failure falls
back to the persistent path (the decoder loads from the store or recomputes).

Counterpart of the reference's RemoteFill stack (lmcache_ascend/v1/
remote_fill.py:272-1694, remote_fill_producer.py:102-1737,
remote_fill_coordinator.py:77-1528, direct_store_plan.py:23-129; wire verbs in
docs/remote_fill_completion_matrix.md:4-6).  The data plane here is the
NVLink push kernel (or a same-process copy for host tests).
"""

from .coordinator import Admission, CircuitBreaker
from .decoder import RemoteFillService
from .planning import plan_windows
from .producer import CopyDataPlane, FillResult, PushDataPlane, RemoteFillProducer

__all__ = ["Admission", "CircuitBreaker", "CopyDataPlane", "FillResult", "PushDataPlane",
           "RemoteFillProducer", "RemoteFillService", "plan_windows"]
