"""The reference's own hot-path tests (its tests/test_page_table.py,
test_prefetch.py, test_archived_runtime.py, test_runtime_spine.py,
test_context_bounds.py, test_exactness_vs_reference.py,
test_generation_restore_continuity.py, test_session_persistence.py and
test_archive_integrity.py) run against the drop-in: ``rfsn_v10_5.cache``,
``.block_manager``, ``.residency`` and ``.storage`` resolve to this
repository's modules (tests/reference_redirect.py) while the reference's
model, layer and attention drive them. CPU only; skipped where the reference
checkout is absent."""

import pytest

from reference_redirect import HOT_PATH_TESTS, reference_available, run_reference_tests

pytestmark = pytest.mark.skipif(not reference_available(), reason="reference checkout not present")


@pytest.mark.parametrize("module_name", HOT_PATH_TESTS)
def test_reference_hot_path_tests_pass_against_the_drop_in(module_name):
    result = run_reference_tests(module_name)
    problems = [f"{t.id()}: {msg.strip().splitlines()[-1]}" for t, msg in result.failures + result.errors]
    assert result.testsRun > 0
    assert not problems, "\n".join(problems)
