"""Record a scheduled child's identity durably, then exec its command.

Reference behaviour: ``src/mimir/scheduling/child.py:1-16``.  Usage:
``python -m mimir_b200.scheduling.child RECEIPT PARENT_PID PARENT_CREATED argv...``.
The receipt (pid + creation time) lets recovery tell a live child from a recycled pid; the
child refuses to start (exit 76) if its parent worker is already gone.
"""
import os
import sys

import psutil

from mimir_b200.evaluation.metrics import write_record

ORPHANED_EXIT = 76


def main(argv) -> None:
    receipt, parent_pid, parent_created, *command = argv
    write_record(receipt, {"pid": os.getpid(), "created": psutil.Process().create_time()})
    try:
        parent = psutil.Process(int(parent_pid))
        alive = parent.create_time() == float(parent_created) and parent.is_running()
    except psutil.NoSuchProcess:
        alive = False
    if not alive:
        sys.exit(ORPHANED_EXIT)
    os.execvpe(command[0], command, os.environ)


if __name__ == "__main__":
    main(sys.argv[1:])
