"""fak_b200: a Blackwell-native (sm_100a) LLM serving engine with an agent-kernel gateway."""
__version__ = "0.1.0"
