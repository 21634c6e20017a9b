"""modded_nanogpt_b200: a Blackwell-native (sm_100a) GPT speedrun training framework."""
__version__ = "0.1.0"
