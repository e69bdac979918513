"""Binding to an externally provided NCCL checkpoint shim (``ncclCheckpointPrepare/Restore``).

Reference behaviour: ``src/mimir/training/suspension/nccl_shim.py:7-29``.  The shim library is
not part of either project; the launcher LD_PRELOADs it and this class resolves the two entry
points from the process image.  Never enabled implicitly.
"""
from __future__ import annotations

import ctypes
import os


class NcclCheckpointShim:
    def __init__(self, library=None):
        if not os.environ.get("NCCL_CHECKPOINT_KVS_PATH"):
            raise RuntimeError("NCCL checkpoint shim requires NCCL_CHECKPOINT_KVS_PATH")
        self.library = ctypes.CDLL(None) if library is None else library
        try:
            self._prepare = self.library.ncclCheckpointPrepare
            self._restore = self.library.ncclCheckpointRestore
        except AttributeError as error:
            raise RuntimeError("NCCL checkpoint shim must be LD_PRELOADed at launch") from error
        for fn in (self._prepare, self._restore):
            fn.argtypes = []
            fn.restype = ctypes.c_int

    def prepare(self) -> None:
        status = self._prepare()
        if status:
            raise RuntimeError(f"ncclCheckpointPrepare failed: NCCL status {status}")

    def restore(self) -> None:
        status = self._restore()
        if status:
            raise RuntimeError(f"ncclCheckpointRestore failed: NCCL status {status}")
