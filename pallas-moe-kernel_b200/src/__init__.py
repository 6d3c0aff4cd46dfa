"""B200 fused MoE expert MLP (sm_100a), laid out like the reference's ``src/``
package so that ``from src.kernel import fused_ragged_dot_caller`` works with
this folder on ``sys.path``."""
