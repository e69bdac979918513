"""Local job scheduler: SQLite queue, worker, idle-GPU coordinator, monitor."""
