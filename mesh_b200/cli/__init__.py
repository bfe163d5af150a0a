"""The ``mesh`` command line."""
