"""A minimal stand-in for the tinygrad package (tests only): the registries that
tinygrad_dx12_b200.compat.register() touches, with the names tinygrad uses."""
