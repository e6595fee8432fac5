"""Logger factory (the reference uses ``lmcache.logging.init_logger``)."""

from __future__ import annotations

import logging
import os
import sys

_FMT = "[%(asctime)s] LMCache-B200 %(levelname)s: %(message)s (%(filename)s:%(lineno)d:%(name)s)"
_configured = False


def init_logger(name: str) -> logging.Logger:
    global _configured
    if not _configured:
        root = logging.getLogger("lmcache_ascend_b200")
        if not root.handlers:
            h = logging.StreamHandler(sys.stderr)
            h.setFormatter(logging.Formatter(_FMT))
            root.addHandler(h)
        root.setLevel(os.environ.get("LMCACHE_LOG_LEVEL", "WARNING").upper())
        root.propagate = False
        _configured = True
    if not name.startswith("lmcache_ascend_b200"):
        name = "lmcache_ascend_b200." + name
    return logging.getLogger(name)
