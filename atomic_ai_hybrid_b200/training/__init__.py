"""Loss, train step and the training loop."""
from .loss import compute_loss, ROUTER_COLLINEARITY_COEF  # noqa: F401
