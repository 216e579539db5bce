/* model forward oracle: filled in below */
