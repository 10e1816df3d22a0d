from maloq_b200.cli.main import main  # noqa: F401

if __name__ == "__main__":
    main()
