"""The exception classes of the batch API (reference tests/test_errors.py): the reference's names,
each also the built-in exception it stands for, library messages mapped onto them, and the option
refusals that need no device."""

import pytest

from cuju_b200 import errors


def test_every_class_is_an_error_and_its_builtin():
    expected = {
        'ConfigurationError': (ValueError,), 'ChoiceError': (ValueError, KeyError), 'ArgumentError': (ValueError,),
        'ActionRangeError': (IndexError,), 'EnvironmentIndexError': (IndexError, RuntimeError),
        'StateError': (ValueError, RuntimeError), 'ClosedError': (RuntimeError,), 'DeviceError': (RuntimeError,),
        'UndefinedPathError': (RuntimeError,), 'LibraryError': (RuntimeError,),
        'MissingFileError': (FileNotFoundError,),
    }
    for name, bases in expected.items():
        cls = getattr(errors, name)
        assert issubclass(cls, errors.Error)
        for base in bases:
            assert issubclass(cls, base), (name, base)
    # KeyError would quote its message; these print it as it is.
    assert str(errors.ChoiceError('no such name')) == 'no such name'


def test_library_messages_map_onto_classes():
    assert type(errors.from_library('an environment reached a path that GRF leaves undefined')) is \
        errors.UndefinedPathError
    assert type(errors.from_library('cuda error in cudaMalloc: out of memory')) is errors.DeviceError
    assert type(errors.from_library('expected an environment from 0 to 3, found 9')) is errors.EnvironmentIndexError
    assert type(errors.from_library('expected a state of the scenario of the environment, found another')) is \
        errors.LibraryError


def test_option_refusals_before_any_device():
    from cuju_b200 import BatchEnvironment

    with pytest.raises(errors.ChoiceError):
        BatchEnvironment('5_vs_5_l4_r0', representation='pixels')
    with pytest.raises(errors.ChoiceError):
        BatchEnvironment('5_vs_5_l4_r0', action_set='mouse')
    with pytest.raises(errors.ConfigurationError):
        BatchEnvironment('5_vs_5_l4_r0', rewards='checkpoints')
    with pytest.raises(errors.ChoiceError):
        BatchEnvironment('5_vs_5_l4_r0', device='cpu')
    from cuju_b200 import resolve_asset

    with pytest.raises(errors.MissingFileError):
        resolve_asset('no_such_scenario_l1_r0')


def test_scenario_name_and_raw_accessors_without_a_device():
    """The names a batch reports and the raw accessors' refusal, on a batch object built without
    a device (only the attributes these read are set)."""
    import pytest

    from cuju_b200 import BatchEnvironment
    from cuju_b200.errors import ConfigurationError

    batch = BatchEnvironment.__new__(BatchEnvironment)
    batch._requested = ['5_vs_5_l4_r0', '/some/dir/academy_attacker_vs_keeper_l0_r0.cjb', '5_vs_5_l4_r0']
    batch._raw = False
    assert batch.scenario_name == '5_vs_5_l4_r0, academy_attacker_vs_keeper_l0_r0'
    with pytest.raises(ConfigurationError):
        batch.raw()
    with pytest.raises(ConfigurationError):
        batch.final_raw()
