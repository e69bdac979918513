"""mimir_b200: a Blackwell-native (sm_100a) training framework for Mimir2 models."""
__version__ = "0.1.0"

from mimir_b200.models import Mimir2, Mimir2Config, LMHead  # noqa: F401
