"""Package logger configured from the ``BRAID_LOG`` environment variable."""
from __future__ import annotations

import logging
import os

_configured = False


def get_logger(name: str = "braidinfer_b200") -> logging.Logger:
    global _configured
    logger = logging.getLogger("braidinfer_b200")
    if not _configured:
        level = os.environ.get("BRAID_LOG", "WARNING").upper()
        logger.setLevel(getattr(logging, level, logging.WARNING))
        if not logger.handlers:
            h = logging.StreamHandler()
            h.setFormatter(logging.Formatter("[braid %(levelname)s] %(message)s"))
            logger.addHandler(h)
        logger.propagate = False
        _configured = True
    return logger if name == "braidinfer_b200" else logger.getChild(name)
