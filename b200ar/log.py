"""Logging for b200ar (level from ``B200AR_LOG_LEVEL``, default WARNING)."""

import logging
import os

logger = logging.getLogger("b200ar")
if not logger.handlers:
    _h = logging.StreamHandler()
    _h.setFormatter(logging.Formatter("[b200ar %(levelname)s] %(message)s"))
    logger.addHandler(_h)
logger.setLevel(os.environ.get("B200AR_LOG_LEVEL", "WARNING").upper())
