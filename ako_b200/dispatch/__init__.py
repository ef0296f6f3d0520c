"""AKO's dispatch interface, re-implemented so the kernels can be selected,
validated and cached where the reference package is not installed.

Same names, arguments, record format and selection rule as the reference's
``ako.dispatcher`` / ``ako.validation`` / ``ako.benchmark`` modules; when the
reference is importable, :func:`ako_b200.plugin.register` registers the CUDA
candidates into the reference's own registry instead.
"""
