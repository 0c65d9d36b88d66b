{
  "targets": [
    {
      "target_name": "hachiue_cuda",
      "sources": ["hachiue_napi.c"],
      "include_dirs": ["../../include"],
      "libraries": ["-L<(module_root_dir)/..", "-lhachiue_cuda", "-Wl,-rpath,<(module_root_dir)/.."],
      "cflags": ["-std=c11", "-O2", "-Wall", "-Wextra"]
    }
  ]
}
