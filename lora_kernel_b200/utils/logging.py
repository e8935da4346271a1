"""Structured JSON-lines logging with the process rank.

Reference: Logger (include/core/logging.hpp:27-102): JSON lines with
{ts, level, logger, file:line, msg, id}; same fields here plus `rank`.
"""
from __future__ import annotations

import itertools
import json
import logging
import os
import sys
import time

_ids = itertools.count()


class JsonFormatter(logging.Formatter):
    def format(self, rec: logging.LogRecord) -> str:
        d = {"ts": round(time.time(), 6), "level": rec.levelname, "logger": rec.name,
             "loc": f"{rec.filename}:{rec.lineno}", "msg": rec.getMessage(), "id": next(_ids),
             "rank": int(os.environ.get("RANK", "0"))}
        extra = getattr(rec, "fields", None)
        if extra:
            d.update(extra)
        return json.dumps(d)


def get_logger(name: str = "lora_kernel", level: str = "INFO", file: str = "") -> logging.Logger:
    log = logging.getLogger(name)
    if not getattr(log, "_lk_configured", False):
        h = logging.StreamHandler(sys.stderr)
        h.setFormatter(JsonFormatter())
        log.addHandler(h)
        if file:
            fh = logging.FileHandler(file)
            fh.setFormatter(JsonFormatter())
            log.addHandler(fh)
        log.propagate = False
        log._lk_configured = True
    log.setLevel(level)
    return log


def log_fields(log: logging.Logger, msg: str, **fields) -> None:
    log.info(msg, extra={"fields": fields})
