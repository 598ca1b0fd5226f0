{
  "targets": [
    {
      "target_name": "qq3",
      "sources": ["qq3_addon.cc"],
      "include_dirs": ["../../include"],
      "libraries": ["-L<(module_root_dir)/..", "-lqq3cuda", "-Wl,-rpath,<(module_root_dir)/.."],
      "cflags_cc": ["-std=c++17", "-O2"]
    }
  ]
}
