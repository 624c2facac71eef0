"""Producer windows cut from a record file (plain and zstd), published atomically and never over an
existing window; the feature pipeline's reader decodes them back to the same records (CPU)."""
import pytest

from flare_b200.data.pipeline import read_chunks
from flare_b200.data.windows import main, read_records, write_stream_windows


def _source(tmp_path, n=40):
    p = tmp_path / "src.txt"
    p.write_text("".join(f"{i}\tuser{i % 7}\titem{i}\n" for i in range(n)))
    return p


@pytest.mark.parametrize("compression", ["plain", "zstd"])
def test_windows_round_trip(tmp_path, compression):
    src = _source(tmp_path)
    out = write_stream_windows(src, tmp_path / "w", rows_per_window=8, windows=3, start_window=1,
                               compression=compression)
    assert [p.name for p in out] == [f"part-0000{k}{'.zst' if compression == 'zstd' else '.txt'}" for k in (1, 2, 3)]
    recs = read_records(src, 32)
    for k, p in zip((1, 2, 3), out):
        assert [r for chunk in read_chunks(str(p), 100) for r in chunk] == recs[8 * k:8 * (k + 1)]
    with pytest.raises(FileExistsError):
        write_stream_windows(src, tmp_path / "w", rows_per_window=8, windows=1, start_window=2,
                             compression=compression)
    assert not [p for p in (tmp_path / "w").iterdir() if p.name.startswith(".")]


def test_windows_need_enough_records(tmp_path, capsys):
    src = _source(tmp_path, 10)
    with pytest.raises(ValueError, match="10 records, 12 needed"):
        write_stream_windows(src, tmp_path / "w", rows_per_window=4, windows=3)
    assert main([str(src), str(tmp_path / "v"), "--rows-per-window", "5", "--windows", "2"]) == 0
    assert "windows=2" in capsys.readouterr().out
