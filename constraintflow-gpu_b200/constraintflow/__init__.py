"""Drop-in replacement of ConstraintFlow's tensor runtime on B200 GPUs.

``constraintflow.gbcsr`` mirrors the reference's block-sparse tensor API with all
arithmetic in libcfgpu; ``constraintflow.lib`` provides the layer-loop entry points
(Flow, abstract element, input spec) that run whole networks through cf_deeppoly_run.
"""
