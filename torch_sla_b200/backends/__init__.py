"""The `pytorch` iterative backend of torch-sla, implemented on B200 kernels."""
from .pytorch_backend import *  # noqa: F401,F403
