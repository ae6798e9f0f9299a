# Stand-in for the `cytoolz` dependency of the reference (absent from this image); only the
# one function the reference imports is provided. Used by make_golden.py only.
