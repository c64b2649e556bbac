"""B200-native LeWM iCEM planning hot path.

Public surface (drop-ins for the reference antoinenguyen27/lewm-flash):

* ``B200ICEMSolver`` -- ``lewm.solvers.icem.ICEMSolver``
* ``B200CEMSolver`` -- ``lewm.solvers.cem_exact.CEMExactSolver``
* ``B200CEMGDSolver`` -- ``lewm.solvers.cem_gd.CEMGDSolver`` (device seed plan + device gradient)
* ``B200ICEMStaticSolver`` -- ``lewm.solvers.icem_static_compile.ICEMStaticCompileSolver``
* ``run_static_icem_chain`` -- ``lewm.solvers.icem_static_compile.run_static_icem_chain``
* ``B200ModelCost`` / ``install_model_cost`` -- ``JEPA.get_cost_from_embeddings``, differentiable
  with respect to the action candidates (float32 reverse pass on the device)
* ``B200Encoder`` / ``install_encoder`` -- ``JEPA.encode`` (ViT CLS row + projector), and
  ``B200Encoder.encode_frames`` for raw uint8 frames (the policy image transform fused)
* ``B200PlanningPolicy`` -- the planning policy the reference evaluates through
  (``get_action``: action buffer, receding-horizon replanning, warm-start tail)
* ``Runtime`` -- the C ABI (``include/lewm_b200.h``) on one GPU

The compute path is ``liblewm_b200.so`` (sm_100a CUDA); there is no CPU
fallback.
"""

from .encoder import B200Encoder, EncoderDesc, install_encoder
from .model import ModelDesc, STRESS_DESC, synthetic_state_dict
from .policy import B200PlanningPolicy
from .runtime import PlanOptions, Runtime, coloring_matrix, sample_counts
from .solver import (B200CEMGDSolver, B200CEMSolver, B200ICEMSolver, B200ICEMStaticSolver, B200ModelCost,
                     install_model_cost, prepare_init_action, run_static_icem_chain)

__all__ = [
    "ModelDesc", "STRESS_DESC", "synthetic_state_dict", "PlanOptions", "Runtime", "coloring_matrix", "sample_counts",
    "B200ICEMSolver", "B200CEMSolver", "B200CEMGDSolver", "B200ICEMStaticSolver", "B200ModelCost", "install_model_cost", "prepare_init_action",
    "run_static_icem_chain", "B200Encoder", "EncoderDesc", "install_encoder",
    "B200PlanningPolicy",
]
