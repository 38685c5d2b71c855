"""Logging setup. VMC_LOG_LEVEL selects the level (the reference uses SPDLOG_LEVEL, src/main.cpp:332)."""
from __future__ import annotations

import logging
import os

_configured = False


def get_logger(name: str) -> logging.Logger:
    global _configured
    if not _configured:
        level = os.environ.get("VMC_LOG_LEVEL", os.environ.get("SPDLOG_LEVEL", "info")).upper()
        logging.basicConfig(level=getattr(logging, level, logging.INFO),
                            format="[%(asctime)s] [%(name)s] [%(levelname)s] %(message)s")
        _configured = True
    return logging.getLogger(f"vmc.{name}")
