"""Model layer: L0 primitives through the complete KimiK3 orchestrator."""
from .attnres import *  # noqa: F401,F403
from .backbone import *  # noqa: F401,F403
from .kda import *  # noqa: F401,F403
from .kimi_k3 import *  # noqa: F401,F403
from .losses import *  # noqa: F401,F403
from .posttrain import *  # noqa: F401,F403
from .mla import *  # noqa: F401,F403
from .moe import *  # noqa: F401,F403
from .mtp import *  # noqa: F401,F403
from .primitives import *  # noqa: F401,F403
from .vision import *  # noqa: F401,F403
from .vision_ablations import *  # noqa: F401,F403
