"""femtotron_b200: a B200-native (sm_100a) 3D-parallel LLaMA pretraining framework."""
__version__ = "0.1.0"
