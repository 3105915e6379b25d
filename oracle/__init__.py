"""FA-KLA oracle (test infrastructure only; never imported by the product).

``oracle.fakla_oracle`` wraps the plain-C restatement in ``fakla_oracle.c``;
``oracle.build_ref`` builds/loads the reference's own CPU kernel into
``oracle/_ref``.
"""
