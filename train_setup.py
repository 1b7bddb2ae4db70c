"""Setup helpers with the reference ``train_setup.py`` roles: model/optimizer/
sharding construction, the apply-step hooks and the multi-source data loader."""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from atomic_ai_hybrid_b200.training.setup import make_shard_and_compile  # noqa: E402,F401
from atomic_ai_hybrid_b200.data import (build_manifest, dataloader_multi_source,  # noqa: E402,F401
                                        resolve_source_files)
from atomic_ai_hybrid_b200.utils.monitor import (NONFINITE_CONSECUTIVE_LIMIT, NONFINITE_WINDOW_RATIO,  # noqa: E402,F401
                                                 NONFINITE_WINDOW_SIZE, SESSION_TIME_BUDGET_SECONDS)
from atomic_ai_hybrid_b200.optim.hybrid import (EXPERT_BIAS_GAMMA, ROUTER_TEMP_DECAY_RATE,  # noqa: E402,F401
                                                ROUTER_TEMP_INIT)
