def thread_first(value, *functions):
    """Apply `functions` to `value` left to right (the only cytoolz call the reference makes)."""
    for fn in functions:
        value = fn(value)
    return value
