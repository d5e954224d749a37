from .ddp import DataParallelGradSync
from .gradient_synchronizer import GradientSynchronizer, NoOpGradSync, create_grad_synchronizer
