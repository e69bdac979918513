from mimir_b200.models.mimir2 import Mimir2, Mimir2Config  # noqa: F401
from mimir_b200.models.lm_head import LMHead  # noqa: F401
