from mimir_b200.config.compose import compose, Composer, ComposeError, MissingValueError  # noqa: F401
