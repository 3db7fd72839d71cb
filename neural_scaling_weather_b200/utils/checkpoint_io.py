"""Checkpoint files that a reader can trust: atomic writes with a SHA-256 record.

A training job can be killed at any moment (preemption, a failing rank), so a checkpoint is
written to a temporary file and renamed into place, and its SHA-256 is kept beside it in
``<file>.sha256``.  Loading checks the record, so a resume never starts from a truncated or
corrupted file.  The checkpoint itself keeps the reference's ``torch.save`` dictionary format
(``utils/trainer.py:755-776`` of the reference); files without a record load unchecked.
"""

from __future__ import annotations

import os

import torch


def _sha256(path: str) -> str:
    import hashlib

    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(8 << 20), b""):
            h.update(block)
    return h.hexdigest()


def atomic_save(obj, path: str) -> None:
    """Write ``obj`` to ``path`` so that a reader never sees a partial file: save to a temporary
    file, record its SHA-256 in ``path + '.sha256'`` (also written atomically), then rename.
    The checkpoint itself keeps the reference's format; the checksum is a separate file."""
    tmp = path + ".tmp"
    torch.save(obj, tmp)
    digest = _sha256(tmp)
    side, side_tmp = path + ".sha256", path + ".sha256.tmp"
    with open(side_tmp, "w") as f:
        f.write(f"{digest}  {os.path.basename(path)}\n")
    os.replace(tmp, path)
    os.replace(side_tmp, side)


def verified_load(path: str, **kwargs):
    """``torch.load`` after checking the file against its ``.sha256`` record when one exists
    (checkpoints written by ``atomic_save``); files without a record (for example the
    reference's own checkpoints) load as they are.  A mismatch raises instead of resuming from
    a truncated or corrupted file."""
    side = path + ".sha256"
    if os.path.exists(side):
        digest = _sha256(path)
        recorded = open(side).read().split()[0]
        if digest != recorded:
            # interrupted between the two renames: the new record is still in its temporary file
            pending = side + ".tmp"
            if os.path.exists(pending) and open(pending).read().split()[0] == digest:
                os.replace(pending, side)
            else:
                raise RuntimeError(f"checkpoint {path} does not match its SHA-256 record ({side}): "
                                   "the file is truncated or corrupted")
    return torch.load(path, **kwargs)
