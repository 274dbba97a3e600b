"""B200 (sm_100a) fused RMSNorm -> Linear, laid out like the reference's ``src``
package so that ``from src.load_cuda import denominator_cuda``,
``from src.fused_forward import FusedRMSNormLinearV3`` and
``from src.weight_transform import compute_fused_weights_rmsnorm`` resolve
here when this project directory is on ``sys.path``.
"""
