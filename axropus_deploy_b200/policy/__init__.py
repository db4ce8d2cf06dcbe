"""Policy layer: state vector, decisions (rules + UCB1 bandit, optional model), safety-clamped
execution, rewards, learned depth policy, a local reasoning model with LoRA adapters and its
learning loop, federated averaging, curricula, and feedback
controllers for batch size. Optional: a worker runs without it."""
from .decide import AdaptivePolicy, Decision, DecisionExecutor, EndpointModel, read_decode_config
from .learn import (REWARD_WEIGHTS, DepthPolicy, FederatedAverager, RewardLedger, RolloutBuffer, adversarial, curriculum,
                    dpo_update, fedavg, ppo_update, reinforce_update, replay_trace)
from .local_model import (LocalReasoningModel, LoRA, LoraLearningLoop, lm_forward, load_adapter, load_peft_adapter,
                          save_peft_adapter)
from .orchestrator import BatchController, Pid, PolicyOrchestrator, power_fraction
from .state import WIDTH, PowerSampler, Slot, StateCollector

__all__ = ["AdaptivePolicy", "Decision", "DecisionExecutor", "EndpointModel", "read_decode_config", "REWARD_WEIGHTS",
           "DepthPolicy", "FederatedAverager", "RewardLedger", "RolloutBuffer", "curriculum", "fedavg", "ppo_update",
           "reinforce_update", "dpo_update", "adversarial", "replay_trace", "BatchController", "Pid", "PolicyOrchestrator", "power_fraction", "WIDTH",
           "PowerSampler", "Slot", "StateCollector", "LocalReasoningModel", "LoRA", "LoraLearningLoop", "lm_forward",
           "load_adapter", "load_peft_adapter", "save_peft_adapter"]
