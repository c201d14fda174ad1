"""Process-wide ``[titan]``-style logger (rank-aware)."""
from __future__ import annotations

import functools
import logging
import os

logger = logging.getLogger("torchtitan_b200")


def init_logger() -> None:
    logger.setLevel(logging.INFO)
    logger.propagate = False
    if not logger.handlers:
        h = logging.StreamHandler()
        rank = os.environ.get("RANK", "0")
        h.setFormatter(logging.Formatter(f"[b200 r{rank}] %(asctime)s %(levelname)s %(message)s"))
        logger.addHandler(h)
    # LOG_RANK="0,1" limits output to those ranks
    allowed = os.environ.get("LOG_RANK")
    if allowed is not None and os.environ.get("RANK", "0") not in allowed.split(","):
        logger.setLevel(logging.WARNING)


@functools.lru_cache(None)
def warn_once(msg: str) -> None:
    logger.warning(msg)
